#!/usr/bin/env python3
"""Generate the golden int8_groupwise vectors in this directory from the reference.

Run where a checkout of the reference is available, giving its path:

    python tests/golden/make_golden_int8.py <reference checkout>
    (or RVQ_REFERENCE_DIR=<reference checkout> python tests/golden/make_golden_int8.py)

Each ``int8_*.npz`` holds an entry produced by the reference's own encoder
``encode_int8_groupwise`` (compress_full_model.py:391-425) -- int8 codes,
fp16 group scales, bf16 tail -- and the reference's own decode
``_decode_int8_into`` (infer_compressed_layerwise_single_slot.py:110-120) of
it into fp16, bf16 and fp32 outputs.
"""

from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("RVQ_REFERENCE_DIR") or (sys.argv[1] if len(sys.argv) > 1 else "")
if not REF or not os.path.isdir(REF):
    sys.exit(f"usage: {os.path.basename(__file__)} <reference checkout> (or set RVQ_REFERENCE_DIR)")
sys.path.insert(0, REF)

import compress_full_model as cfm  # noqa: E402  (reference)
import infer_compressed_layerwise_single_slot as ss  # noqa: E402  (reference)

ss.torch = torch
OUT_DTYPES = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}


def bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.float32:
        return t.contiguous().view(torch.int32).numpy().view(np.uint32).reshape(-1)
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).reshape(-1)


def save_case(name, w, group_size, note):
    entry = cfm.encode_int8_groupwise(w, group_size)
    assert entry["method"] == "int8_groupwise", name
    arrays = {
        "q": entry["q"].numpy().reshape(-1),
        "scales_f16": bits(entry["scales"]),
        "tail_bf16": bits(entry["tail"]),
    }
    for key, dt in OUT_DTYPES.items():
        out = torch.zeros(tuple(entry["shape"]), dtype=dt)
        ss._decode_int8_into(entry, out)
        arrays[f"expected_{key}"] = bits(out)
    meta = {"shape": list(entry["shape"]), "group_size": int(entry["group_size"]),
            "trimmed_numel": int(entry["trimmed_numel"]), "method": entry["method"], "note": note}
    arrays["meta_json"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrays)
    print(f"{name}: shape={meta['shape']} group={group_size} trimmed={meta['trimmed_numel']} "
          f"tail={entry['tail'].numel()}")


def main():
    g = torch.Generator().manual_seed(70)
    save_case("int8_g128", torch.randn(64, 256, generator=g) * 0.02, 128, "group 128, no tail")
    save_case("int8_tail", torch.randn(37, 100, generator=g) * 0.02, 128, "numel % group_size != 0 -> bf16 tail")
    save_case("int8_g16", torch.randn(48, 64, generator=g) * 0.05, 16, "group 16")
    save_case("int8_g7", torch.randn(13, 29, generator=g), 7, "group 7: groups straddle 16-element lanes, tail 6")
    w = torch.randn(40, 128, generator=g) * 0.02
    w[0] = 0.0                                   # all-zero group: scale clamped to 1e-8 / 127
    w[1, :64] = 1.0e7                            # fp16 scale overflows to inf: q * inf, 0 * inf = nan
    w[2, 5] = 70000.0                            # one large value per group
    save_case("int8_extreme", w, 64, "zero group, fp16-overflowing scale, outlier")
    save_case("int8_big", torch.randn(300, 517, generator=g) * 0.02, 128, "155100 elements, tail 92")


if __name__ == "__main__":
    main()
