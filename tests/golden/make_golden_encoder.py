#!/usr/bin/env python3
"""Golden vectors for the GPU encoder from the reference's own compressor.

Run where a checkout of the reference is available, giving its path:

    python tests/golden/make_golden_encoder.py <reference checkout>
    (or RVQ_REFERENCE_DIR=<reference checkout> python tests/golden/make_golden_encoder.py)

Writes ``encoder_cases.npz``:
* ``assign_*``: 20000 vectors, a 256-code codebook, the reference's
  assign_codes (compress_full_model.py:202-208) and, per vector, the gap
  between its best and second-best pairwise_sqdist distance (lines 196-199);
* ``kmeans_*``: 30000 vectors, the reference's kmeans_train (lines 211-234)
  with k=64, 4 iterations, seed 7, and the mean squared error of assigning
  the vectors to its centroids;
* ``enc_*``: a [96, 512] weight, codebooks trained by the reference's residual
  k-means on its normalised vectors, and the reference's encode_rvq_tensor
  (lines 337-388) entry at group size 128: codes, fp16 scales, mse, rel_rmse.
"""

from __future__ import annotations

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


def main():
    torch.manual_seed(0)
    g = torch.Generator().manual_seed(80)
    out = {}
    x = torch.randn(20000, 8, generator=g) * 0.3
    c = torch.randn(256, 8, generator=g) * 0.3
    idx = cfm.assign_codes(x, c, chunk_size=4096)
    d = cfm.pairwise_sqdist(x, c)
    two = torch.topk(d, 2, dim=1, largest=False).values
    out.update(assign_x=x.numpy(), assign_c=c.numpy(), assign_idx=idx.numpy(),
               assign_gap=(two[:, 1] - two[:, 0]).numpy())

    xk = torch.randn(30000, 8, generator=g) * torch.linspace(0.2, 1.0, 8)
    cent = cfm.kmeans_train(xk, k=64, iters=4, seed=7, chunk_size=8192)
    a = cfm.assign_codes(xk, cent, chunk_size=8192)
    mse = float(((xk - cent[a]) ** 2).sum(dim=1).mean())
    out.update(kmeans_x=xk.numpy(), kmeans_centroids=cent.numpy(), kmeans_mse=np.float64(mse))

    w = torch.randn(96, 512, generator=g) * 0.02
    norm, _, _ = cfm.normalize_groups(w.view(-1), 128)
    v = cfm.to_vectors(norm, 8)
    residual, cbs = v.clone(), []
    for r in range(4):
        cb = cfm.kmeans_train(residual, k=256, iters=4, seed=90 + 31 * r, chunk_size=8192)
        residual = residual - cb[cfm.assign_codes(residual, cb, chunk_size=8192)]
        cbs.append(cb)
    cbs = torch.stack(cbs, 0).to(torch.float16).contiguous()
    e = cfm.encode_rvq_tensor(w, cbs, d=8, group_size=128, chunk_size=8192, codebook_id="fixture")
    out.update(enc_w=w.numpy(), enc_codebooks=cbs.view(torch.int16).numpy(), enc_codes=e["indices"].numpy(),
               enc_scales=e["scales"].view(torch.int16).numpy(), enc_mse=np.float64(e["mse"]),
               enc_rel_rmse=np.float64(e["rel_rmse"]))
    np.savez_compressed(os.path.join(HERE, "encoder_cases.npz"), **out)
    print("assign: near ties (gap < 1e-6):", int((out["assign_gap"] < 1e-6).sum()),
          "kmeans mse", mse, "encode rel_rmse", e["rel_rmse"])


if __name__ == "__main__":
    main()
