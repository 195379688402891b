"""GPU encoder throughput on the config-0 matrix.

    python -m rvq_b200.bench_encode

Encodes a seeded [9728, 2560] N(0, 0.02) weight with 4 stages x 256 codes
(group size 2560, d = 8: 3,112,960 vectors) through
``rvq_b200.encoder.encode_rvq_tensor``, and runs ``kmeans_train`` (k = 256,
4 iterations) on 1,048,576 vectors.  Device time by CUDA events after one
untimed run.  Prints one JSON object.
"""

from __future__ import annotations

import json

import torch

from . import encoder, synthetic


def _time(fn):
    fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    out = fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e), out


def run(device="cuda:0"):
    device = torch.device(device)
    torch.cuda.set_device(device)
    g = torch.Generator(device=device).manual_seed(0)
    w = torch.randn(9728, 2560, generator=g, device=device) * 0.02
    cbs = synthetic.make_codebook(4, 256, 8, torch.Generator().manual_seed(1)).to(device)
    ms_enc, e = _time(lambda: encoder.encode_rvq_tensor(w, cbs, 8, 2560, 65536, "bench"))
    nvec = w.numel() // 8
    x = torch.randn(1 << 20, 8, generator=g, device=device) * 0.3
    ms_km, _ = _time(lambda: encoder.kmeans_train(x, 256, 4, 0))
    return {"encode": {"workload": "[9728, 2560] weight, 4 x 256 codes, d=8, group 2560", "ms": round(ms_enc, 3),
                       "vectors_per_s": round(nvec / ms_enc * 1e3, 1),
                       "distance_evaluations_per_s": round(nvec * 4 * 256 / ms_enc * 1e3, 1),
                       "rel_rmse": round(e["rel_rmse"], 5)},
            "kmeans": {"workload": "1,048,576 vectors, k=256, 4 iterations", "ms": round(ms_km, 3)},
            "timing": "CUDA events around one call after an untimed call (includes the host-side tensor ops)"}


def main():
    print(json.dumps(run()))


if __name__ == "__main__":
    main()
