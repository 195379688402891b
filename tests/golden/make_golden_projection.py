#!/usr/bin/env python3
"""A golden entry at a real projection shape and the compressor's default
group size, from the reference itself.

Run where a checkout of the reference is available, giving its path:

    python tests/golden/make_golden_projection.py <reference checkout>
    (or RVQ_REFERENCE_DIR=<reference checkout> python tests/golden/make_golden_projection.py)

A seeded [1024, 2560] N(0, 0.02) weight (the k_proj shape of the
2560-hidden block) is encoded by the reference's own pipeline: residual
k-means codebooks (kmeans_train / assign_codes on 65,536 of its normalised
vectors, compress_full_model.py:204-234, 325-334) and encode_rvq_tensor at
group_size=128 (the default of compress_full_model.py:459; lines 337-388).
``proj_k_g128.npz`` holds the entry (uint8 code planes, fp16 scales, fp16
codebooks) and the sha256 of the reference's _decode_rvq_into output
(infer_compressed_layerwise_single_slot.py:123-149) in fp16, bf16 and fp32.
"""

from __future__ import annotations

import hashlib
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


def main():
    torch.manual_seed(0)
    g = torch.Generator().manual_seed(2024)
    w = torch.randn(1024, 2560, generator=g) * 0.02
    norm, _, _ = cfm.normalize_groups(w.view(-1), 128)
    v = cfm.to_vectors(norm, 8)
    sample = v[torch.randperm(v.shape[0], generator=g)[:65536]]
    residual, cbs = sample.clone(), []
    for r in range(4):
        cb = cfm.kmeans_train(residual, k=256, iters=4, seed=300 + 31 * r, chunk_size=65536)
        residual = residual - cb[cfm.assign_codes(residual, cb, chunk_size=65536)]
        cbs.append(cb)
    cbs = torch.stack(cbs, 0).to(torch.float16).contiguous()
    e = cfm.encode_rvq_tensor(w, cbs, d=8, group_size=128, chunk_size=65536, codebook_id="attn_k_proj")
    out = {"indices": e["indices"].numpy(), "scales_f16": e["scales"].view(torch.int16).numpy(),
           "codebook_f16": cbs.view(torch.int16).numpy(), "rel_rmse": np.float64(e["rel_rmse"])}
    for key, dt in (("f16", torch.float16), ("bf16", torch.bfloat16), ("f32", torch.float32)):
        o = torch.zeros(1024, 2560, dtype=dt)
        ss._decode_rvq_into(e, cbs.to(torch.float32), o)
        b = o.view(torch.int32 if dt == torch.float32 else torch.int16).numpy().tobytes()
        out[f"sha256_{key}"] = np.frombuffer(hashlib.sha256(b).hexdigest().encode(), dtype=np.uint8)
    np.savez_compressed(os.path.join(HERE, "proj_k_g128.npz"), **out)
    print("rel_rmse", e["rel_rmse"], "indices", e["indices"].shape, e["indices"].dtype)


if __name__ == "__main__":
    main()
