#!/usr/bin/env python3
"""Generate the golden RVQ vectors in this directory from the reference itself.

Run where a checkout of the reference is available, giving its path:

    python tests/golden/make_golden.py <reference checkout>
    (or RVQ_REFERENCE_DIR=<reference checkout> python tests/golden/make_golden.py)

What it records
* ``<case>.npz``: an entry (indices, codebook, scales, tail, metadata) and
  the reference's decoded output for fp16, bf16 and fp32, produced by
  ``_decode_rvq_into`` (infer_compressed_layerwise_single_slot.py:123-149).
  The ``enc_*`` cases are encoded by the reference's own ``kmeans_train``,
  ``assign_codes`` and ``encode_rvq_tensor`` (compress_full_model.py:204-234,
  337-388); the ``syn_*`` cases are hand-built edge cases (K = 1/2/3, int16
  indices with 512 codes, a single vector, ragged vector counts, -0.0
  codewords, fp16 overflow and subnormals, a codebook that fp16 cannot hold
  exactly, trimmed_numel below nvec * d).
* ``checksums.json``: sha256 of the reference's output for the full-size
  seeded workloads (the [9728, 2560] matrix, and the 7 projections of one
  2560/9728 block), which are too large to commit as arrays.

The reference's single_slot engine loads its runtime lazily and needs the
absent ``accelerate`` package for that, so this script sets the module-global
``torch`` that ``_decode_rvq_into`` reads and calls the function directly.
"""

from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("RVQ_REFERENCE_DIR") or (sys.argv[1] if len(sys.argv) > 1 else "")
if not REF or not os.path.isdir(REF):
    sys.exit(f"usage: {os.path.basename(__file__)} <reference checkout> (or set RVQ_REFERENCE_DIR)")
sys.path.insert(0, REF)
sys.path.insert(0, REPO)

import compress_full_model as cfm  # noqa: E402  (reference)
import infer_compressed_layerwise_single_slot as ss  # noqa: E402  (reference)

from rvq_b200 import synthetic  # noqa: E402

ss.torch = torch

OUT_DTYPES = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}


def ref_decode(entry, codebook, dtype):
    out = torch.zeros(tuple(entry["shape"]), dtype=dtype)
    ss._decode_rvq_into(entry, codebook.to(torch.float32), out)
    return out


def bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.float32:
        return t.contiguous().view(torch.int32).numpy().view(np.uint32).reshape(-1)
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).reshape(-1)


def save_case(name, entry, codebook, note):
    arrays = {
        "indices": entry["indices"].numpy(),
        "scales_f16": bits(entry["scales"].to(torch.float16)),
        "tail_bf16": bits(entry["tail"].to(torch.bfloat16)),
    }
    if codebook.dtype == torch.float16:
        arrays["codebook_f16"] = bits(codebook).reshape(codebook.shape)
    else:
        arrays["codebook_f32"] = bits(codebook.to(torch.float32)).reshape(codebook.shape)
    for key, dt in OUT_DTYPES.items():
        arrays[f"expected_{key}"] = bits(ref_decode(entry, codebook, dt))
    meta = {
        "shape": list(entry["shape"]), "group_size": int(entry["group_size"]),
        "d": int(entry["d"]), "trimmed_numel": int(entry["trimmed_numel"]),
        "method": entry["method"], "note": note,
    }
    arrays["meta_json"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrays)
    print(f"{name}: shape={meta['shape']} K={entry['indices'].shape[0]} "
          f"nvec={entry['indices'].shape[1]} tail={entry['tail'].numel()}")


def train_codebooks(x: torch.Tensor, stages: int, k: int, seed: int) -> torch.Tensor:
    """Residual k-means exactly as train_shared_rvq_codebooks' inner loop
    (compress_full_model.py:325-334), using the reference's own functions."""
    residual = x.clone()
    cbs = []
    for r in range(stages):
        cb = cfm.kmeans_train(residual, k=k, iters=4, seed=seed + 31 * r, chunk_size=65536)
        idx = cfm.assign_codes(residual, cb, chunk_size=65536)
        residual = residual - cb[idx]
        cbs.append(cb)
    return torch.stack(cbs, 0).to(torch.float16).contiguous()


def encoded_case(name, shape, group_size, stages, k, seed, note):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(shape, generator=g) * 0.02
    norm, _, _ = cfm.normalize_groups(w.view(-1), group_size)
    x = cfm.to_vectors(norm, 8)
    cb = train_codebooks(x, stages, k, seed)
    entry = cfm.encode_rvq_tensor(w, cb, d=8, group_size=group_size, chunk_size=65536,
                                  codebook_id="fixture")
    save_case(name, entry, cb, note)


def synthetic_case(name, shape, group_size, stages, ncodes, seed, note, mutate=None,
                   codebook=None):
    g = torch.Generator().manual_seed(seed)
    cb = codebook if codebook is not None else synthetic.make_codebook(stages, ncodes, 8, g)
    entry = synthetic.make_rvq_entry(shape[0], shape[1], g, stages=stages, ncodes=ncodes,
                                     group_size=group_size, codebook_id="fixture")
    if mutate is not None:
        entry, cb = mutate(entry, cb)
    save_case(name, entry, cb, note)


def main():
    torch.manual_seed(0)
    encoded_case("enc_g128", (64, 256), 128, 4, 256, 11, "reference encoder, group 128")
    encoded_case("enc_tail", (37, 100), 128, 4, 256, 12, "numel % group_size != 0 -> bf16 tail")
    encoded_case("enc_rowscale", (48, 320), 320, 4, 256, 13, "per-row scales (group = in_features)")
    encoded_case("enc_g8", (64, 64), 8, 2, 256, 14, "one scale per vector, K=2")

    synthetic_case("syn_k1", (24, 96), 32, 1, 256, 21, "K=1")
    synthetic_case("syn_k3_int16", (40, 160), 160, 3, 512, 22, "int16 indices, 512 codes")
    synthetic_case("syn_one_vector", (1, 8), 8, 4, 256, 23, "a single vector")
    synthetic_case("syn_ragged", (1037, 8), 128, 4, 256, 24, "nvec=1037: no block multiple")
    synthetic_case("syn_ragged_tail", (131, 29), 64, 4, 256, 25, "ragged, tail of 23")
    synthetic_case("syn_k2_g16", (256, 48), 16, 2, 256, 26, "K=2, group 16")

    def negzero(entry, cb):
        cb = cb.clone()
        cb[:, 7, :4] = -0.0                       # every stage: -0.0 in lanes 0..3
        entry["indices"][:, :64] = 7
        return entry, cb
    synthetic_case("syn_negzero", (32, 64), 64, 4, 256, 27, "-0.0 in every stage -> +0.0", negzero)

    def extreme(entry, cb):
        cb = cb.clone()
        cb[0, 0] = 60000.0                        # * scale 1.5 overflows fp16 -> inf
        cb[0, 1] = 3.0e-8                         # fp16 subnormal range after scaling
        cb[1, 2] = -65504.0
        entry["indices"][0, ::5] = 0
        entry["indices"][0, 1::5] = 1
        entry["indices"][1, 2::7] = 2
        entry["scales"] = torch.full_like(entry["scales"], 1.5)
        return entry, cb
    synthetic_case("syn_extreme", (16, 128), 128, 2, 256, 28, "fp16 overflow / subnormal", extreme)

    g = torch.Generator().manual_seed(29)
    cb32 = torch.randn(4, 256, 8, generator=g) * 0.02          # not representable in fp16
    synthetic_case("syn_cb_f32", (64, 128), 128, 4, 256, 29, "fp32 codebook (not fp16-exact)",
                   codebook=cb32)

    def trimmed_short(entry, cb):
        entry["trimmed_numel"] = int(entry["trimmed_numel"]) - 5
        entry["tail"] = torch.full((5,), 0.25, dtype=torch.bfloat16)
        return entry, cb
    synthetic_case("syn_trimmed_short", (8, 64), 64, 4, 256, 30,
                   "trimmed_numel = nvec*d - 5 (masked core, tail behind it)", trimmed_short)

    checksums = {}
    entry, cb = synthetic.make_config0_entry(seed=0)
    out = ref_decode(entry, cb, torch.float16)
    checksums["config0_seed0_f16"] = hashlib.sha256(bits(out).tobytes()).hexdigest()
    print("config0", checksums["config0_seed0_f16"])
    art = synthetic.make_block_artifact(seed=0)
    for key, e in art["entries"].items():
        if e["method"] != "rvq_groupwise":
            continue
        o = ref_decode(e, art["shared_codebooks"][e["codebook_id"]], torch.bfloat16)
        checksums[f"block_seed0_bf16:{key}"] = hashlib.sha256(bits(o).tobytes()).hexdigest()
        print(key, checksums[f"block_seed0_bf16:{key}"][:16])
    with open(os.path.join(HERE, "checksums.json"), "w") as f:
        json.dump(checksums, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
