"""Linear-layer microbenchmark on the [9728 x 2560] gate projection.

    python -m rvq_b200.bench_linear [--reps 200] [--batches 1,8,64,2048] [--only fused_tc,dense]

Times device work per call -- each measured loop is captured in a CUDA graph
and the replay timed with CUDA events, so host launch cost is excluded --
with weights rotated over 16 resident copies (no copy's codes stay in L2
between uses):

* ``fused``:  rvq_gemv / rvq_gemv_tiles (batch 1, table GEMV) and
  rvq_gemv_tiles_exact (bit-exact bf16 weights), W never materialised;
* ``fused_tc``: rvq_gemv_batch, W decoded into tensor memory as the tcgen05
  MMA's A operand (every batch size, and the 2048-token prefill); fp16 stage
  sums, and ``fused_tc_exact`` with bit-exact bf16 weights;
* ``decode+gemm``: rvq_decode_layer into a bf16 slot, then torch.matmul
  (cuBLAS) -- the reference's dataflow (infer_compressed_layerwise_triton.py:
  263, 290-292);
* ``dense``: torch.matmul on a resident bf16 weight (the uncompressed model);

at batch 1, 8, 64 and a 2048-token prefill.  Prints one JSON object.
"""

from __future__ import annotations

import argparse
import json

import torch

from . import synthetic
from .engine import LayerDecodePlan
from .gemm import BatchGemvPlan, GemmPlan
from .gemv import GemvPlan, GemvTilesPlan, interleave_codes, tile_codes, tiles_count

ROWS, COLS = 9728, 2560
COPIES = 16


def _time(fn, reps, stream):
    """Device time per call: ``reps`` calls captured in one CUDA graph,
    replayed after a warm-up replay, timed with events (no host launch cost
    in the measurement)."""
    for i in range(3):
        fn(i)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(reps):
            fn(i)
    graph.replay()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    graph.replay()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / reps * 1e3      # us


def run(reps: int = 200, device="cuda:0", batches=(1, 8, 64, 2048), only=None):
    """``batches``: token counts of the batched cases; ``only``: names of the
    cases to run (prefixes such as ``fused_tc``), all when None."""
    want = lambda name: only is None or any(name.startswith(o) for o in only)
    device = torch.device(device)
    torch.cuda.set_device(device)
    g = torch.Generator().manual_seed(0)
    cb = synthetic.make_codebook(4, 256, 8, g)
    entry = synthetic.make_rvq_entry(ROWS, COLS, g, codebook_id="mlp_gate_proj")
    cbd = cb.to(device, torch.float32)
    copies = [{k: (v.to(device) if torch.is_tensor(v) else v) for k, v in entry.items()} for _ in range(COPIES)]
    stream = torch.cuda.current_stream(device)
    out = {"workload": "gate projection [9728 x 2560], K=4, 256 codes, d=8, per-row fp16 scales, bf16 activations",
           "weights_rotated": COPIES, "results": {}}
    code_bytes = copies[0]["indices"].numel() + copies[0]["scales"].numel() * 2

    # fused GEMV, batch 1
    x1 = torch.randn(COLS, generator=g).to(device, torch.bfloat16)
    ys = [torch.empty(ROWS, dtype=torch.bfloat16, device=device) for _ in range(COPIES)]
    algo = code_bytes + COLS * 2 + ROWS * 2
    if want("fused_b1_planes"):
        plans = [GemvPlan([(c, cbd, x1, y)]) for c, y in zip(copies, ys)]
        t = _time(lambda i: plans[i % COPIES].launch(), reps, stream)
        out["results"]["fused_b1_planes"] = {"us": round(t, 2), "GB/s": round(algo / t / 1e3, 1),
                                             "algorithmic_bytes": algo}
    il = [dict(c, codes_il=interleave_codes(c["indices"])) for c in copies]
    if want("fused_b1"):
        plans = [GemvPlan([(c, cbd, x1, y)]) for c, y in zip(il, ys)]
        t = _time(lambda i: plans[i % COPIES].launch(), reps, stream)
        out["results"]["fused_b1"] = {"us": round(t, 2), "GB/s": round(algo / t / 1e3, 1),
                                      "algorithmic_bytes": algo, "codes": "interleaved"}

    # per-tile partials (the form the decode step consumes), and with the tile sum
    parts = [torch.empty(tiles_count(COLS), ROWS, dtype=torch.float32, device=device) for _ in range(COPIES)]
    tl = [dict(c, codes_tiled=tile_codes(c["indices"], ROWS, COLS)) for c in copies]
    tplans = [GemvTilesPlan([(c, cbd, x1, p)]) for c, p in zip(tl, parts)]
    if want("fused_tiles_b1"):
        t = _time(lambda i: tplans[i % COPIES].launch(), reps, stream)
        out["results"]["fused_tiles_b1"] = {"us": round(t, 2), "GB/s": round(algo / t / 1e3, 1),
                                            "algorithmic_bytes": algo, "output": "fp32 partials [10, rows]"}
    if want("fused_exact_tiles_b1"):
        eplans = [GemvTilesPlan([(c, cbd, x1, p)], exact=True) for c, p in zip(tl, parts)]
        t = _time(lambda i: eplans[i % COPIES].launch(), reps, stream)
        out["results"]["fused_exact_tiles_b1"] = {"us": round(t, 2), "GB/s": round(algo / t / 1e3, 1),
                                                  "output": "fp32 partials, bit-exact bf16 weights"}
    y1 = torch.empty(ROWS, dtype=torch.float32, device=device)

    def tiles_sum(i):
        tplans[i % COPIES].launch()
        torch.sum(parts[i % COPIES], 0, out=y1)

    if want("fused_tiles_b1+sum"):
        t = _time(tiles_sum, reps, stream)
        out["results"]["fused_tiles_b1+sum"] = {"us": round(t, 2)}

    # decode + GEMM (slot then cuBLAS), and dense
    need_dense = any(want(f"{n}_b{b}") for n in ("decode+gemm", "dense") for b in batches) or want("decode_only")
    slot = torch.empty(ROWS, COLS, dtype=torch.bfloat16, device=device)
    dplans = [LayerDecodePlan([("w", c)], {"mlp_gate_proj": cbd}, {"w": slot}) for c in copies]
    dense = []
    if need_dense:
        for i in range(COPIES):
            dplans[i].launch(stream.cuda_stream)
            dense.append(slot.clone())
    if want("decode_only"):
        t_dec = _time(lambda i: dplans[i % COPIES].launch(), reps, stream)
        out["results"]["decode_only"] = {"us": round(t_dec, 2)}
    for b in batches:
        x = torch.randn(b, COLS, generator=g).to(device, torch.bfloat16)

        y_dg = torch.empty(b, ROWS, dtype=torch.bfloat16, device=device)
        y_dn = torch.empty(b, ROWS, dtype=torch.bfloat16, device=device)

        def dec_gemm(i, x=x, y=y_dg):
            dplans[i % COPIES].launch()
            torch.matmul(x, slot.t(), out=y)

        def dense_mm(i, x=x, y=y_dn):
            torch.matmul(x, dense[i % COPIES].t(), out=y)

        r = reps if b < 2048 else max(20, reps // 10)
        flops = 2.0 * b * ROWS * COLS
        for exact in (False, True):
            name = f"fused_tc{'_exact' if exact else ''}_b{b}"
            if want(name):
                # the tensor-core fused GEMM (W decoded on chip, never to HBM)
                y_fb = torch.empty(b, ROWS, dtype=torch.bfloat16, device=device)
                bplans = [BatchGemvPlan(c, cbd, x, y_fb, exact=exact) for c in tl]
                t_fb = _time(lambda i: bplans[i % COPIES].launch(), r, stream)
                out["results"][name] = {"us": round(t_fb, 2), "TFLOP/s": round(flops / t_fb / 1e6, 2),
                                        "GB/s": round((code_bytes + b * (COLS + ROWS) * 2) / t_fb / 1e3, 1)}
                del bplans
        if b >= 64 and want(f"fused_gemm_b{b}"):
            # prefill-style: weight decoded into shared memory feeding tcgen05 MMAs
            y_fg = torch.empty(b, ROWS, dtype=torch.bfloat16, device=device)
            gplans = [GemmPlan(c, cbd, x, y_fg) for c in il]
            t_fg = _time(lambda i: gplans[i % COPIES].launch(), r, stream)
            out["results"][f"fused_gemm_b{b}"] = {"us": round(t_fg, 2),
                                                  "TFLOP/s": round(2.0 * b * ROWS * COLS / t_fg / 1e6, 2)}
        if want(f"decode+gemm_b{b}"):
            t_dg = _time(dec_gemm, r, stream)
            out["results"][f"decode+gemm_b{b}"] = {"us": round(t_dg, 2), "TFLOP/s": round(flops / t_dg / 1e6, 2)}
        if want(f"dense_b{b}"):
            t_dn = _time(dense_mm, r, stream)
            out["results"][f"dense_b{b}"] = {"us": round(t_dn, 2), "TFLOP/s": round(flops / t_dn / 1e6, 2),
                                             "GB/s": round((ROWS * COLS * 2 + b * (COLS + ROWS) * 2) / t_dn / 1e3,
                                                           1)}
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reps", type=int, default=200)
    ap.add_argument("--batches", default="1,8,64,2048", help="token counts of the batched cases")
    ap.add_argument("--only", default=None, help="comma-separated case-name prefixes to run (default: all)")
    a = ap.parse_args()
    print(json.dumps(run(a.reps, batches=tuple(int(b) for b in a.batches.split(",")),
                         only=a.only.split(",") if a.only else None)))


if __name__ == "__main__":
    main()
