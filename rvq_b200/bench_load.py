"""Artifact load: the reference's torch.load + per-tensor upload against the
native pack loader.

    python -m rvq_b200.bench_load [--layers 8] [--dir /tmp]

Model: the 2560 / 9728 / 32q / 8kv / 128 block x ``layers``, vocab 151936
(tied bf16 embedding), K=4 256-code RVQ projections, written once with
torch.save (as compress_full_model.py:624-631 does) and once as a pack.
Timed, each after one untimed load so both read from the page cache:
* reference: ``torch.load(path)`` then ``.to(device)`` of every tensor
  (infer_compressed_layerwise_triton.py:421-432), synchronised;
* pack: ``rvq_b200.pack.read_pack`` (one device buffer, rvq_pack_load).
Prints one JSON object (seconds and GB/s of artifact bytes).
"""

from __future__ import annotations

import argparse
import json
import os
import tempfile
import time

import torch

from . import pack, synthetic


def _reference_load(path, device):
    art = torch.load(path, map_location="cpu", weights_only=False)
    cbs = {k: v.to(device) for k, v in art["shared_codebooks"].items()}
    ents = {k: {f: (v.to(device, non_blocking=False) if torch.is_tensor(v) else v) for f, v in e.items()}
            for k, e in art["entries"].items()}
    torch.cuda.synchronize(device)
    return cbs, ents


def run(layers=8, vocab=151936, directory=None, device="cuda:0"):
    device = torch.device(device)
    torch.cuda.set_device(device)
    art = synthetic.make_model_artifact(synthetic.BlockShape(), layers, vocab, seed=0)
    nbytes = sum(v.numel() * v.element_size() for e in art["entries"].values() for v in e.values()
                 if torch.is_tensor(v)) + sum(v.numel() * v.element_size() for v in art["shared_codebooks"].values())
    d = directory or tempfile.gettempdir()
    pt, pk = os.path.join(d, "rvq_bench_artifact.pt"), os.path.join(d, "rvq_bench_artifact.rvqpack")
    torch.save(art, pt)
    pack.write_pack(art, pk)
    del art
    out = {"workload": f"2560/9728 block x {layers} layers + vocab {vocab} embedding, RVQ artifact",
           "artifact_bytes": nbytes}
    for name, fn in (("reference_torch_load", lambda: _reference_load(pt, device)),
                     ("pack_native", lambda: pack.read_pack(pk, device))):
        r = fn()                                  # untimed: page cache, allocator, CUDA context
        del r
        torch.cuda.synchronize(device)
        t = time.perf_counter()
        r = fn()
        torch.cuda.synchronize(device)
        el = time.perf_counter() - t
        del r
        torch.cuda.empty_cache()
        out[name] = {"seconds": round(el, 3), "GB/s": round(nbytes / el / 1e9, 2)}
    for p in (pt, pk):
        os.unlink(p)
    out["speedup"] = round(out["reference_torch_load"]["seconds"] / out["pack_native"]["seconds"], 2)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--dir", default=None)
    a = ap.parse_args()
    print(json.dumps(run(a.layers, directory=a.dir)))


if __name__ == "__main__":
    main()
