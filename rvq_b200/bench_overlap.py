"""Config-1 overlap: decoding the next layer into the other slot while a bf16
block forward runs on a [1, 2560] activation.

    python -m rvq_b200.bench_overlap [--reps 50]

The forward is the native batch-1 decode step of a 2-layer model of the
2560/9728/32q/8kv/128 block with resident bf16 weights (vocab 256, so the
head is negligible), replayed from its CUDA graph; the decode is one
``rvq_decode_layer`` launch per layer into a bf16 slot (the reference's
``prefetch_layer`` side-stream fill, infer_compressed_layerwise_triton.py:
246-266).  Reported: t_fwd and t_dec per layer alone, t_both with the decode
on a side stream concurrent with the forward, overlap =
(t_dec + t_fwd - t_both) / min(t_dec, t_fwd) (1 = the decode is hidden
completely, 0 = the two serialise), the decode GB/s alone and the time the
decode still adds per layer when overlapped.  Prints one JSON object.
"""

from __future__ import annotations

import argparse
import json

import torch

from . import synthetic
from .decoder import Qwen3Decoder
from .engine import LayerDecodePlan
from .slots import SlotArena, SlotSpec


def run(reps: int = 50, device="cuda:0", max_ctas: int = 0, forward_mode: str = "dense"):
    """``max_ctas``: CTA budget of the decode launches (0: one per SM);
    ``forward_mode``: weight mode of the forward decoder ("dense": bf16
    weights as a decoded slot holds them, cuBLAS; "fused": the table GEMV).
    The forward runs on a high-priority stream, the decode on a low-priority
    side stream, as a ping-pong engine would arrange them."""
    device = torch.device(device)
    torch.cuda.set_device(device)
    shape = synthetic.BlockShape()
    art = synthetic.make_model_artifact(shape, 2, 256, seed=3)
    cfg = synthetic.qwen3_config(shape, 2, 256)
    dec = Qwen3Decoder(cfg, art, device, mode=forward_mode, max_len=64)
    dec.capture()
    dec.prefill(torch.arange(8, device=device))
    fwd_graph = dec.graph

    # decode side: 4 further layers rotating over 2 slots (inputs > L2)
    gen = torch.Generator().manual_seed(4)
    cbs = {k: v.to(device, torch.float32) for k, v in synthetic.make_family_codebooks(gen).items()}
    layers = []
    for l in range(4):
        ents = synthetic.make_block_entries(shape, l, gen)
        layers.append({k.split(f"layers.{l}.")[1]: {ek: (ev.to(device) if torch.is_tensor(ev) else ev)
                                                   for ek, ev in e.items()} for k, e in ents.items()})
    names = list(layers[0].keys())
    specs = [[SlotSpec(n, tuple(int(s) for s in layers[l][n]["shape"]), torch.bfloat16) for n in names]
             for l in range(4)]
    arena = SlotArena(specs, device)
    plans = [LayerDecodePlan(list(layers[l].items()), cbs, arena.views(l), max_ctas=max_ctas) for l in range(4)]
    algo = plans[0].algorithmic_bytes

    lo, hi = torch.cuda.Stream.priority_range()            # (lowest, greatest) priority
    main, side = torch.cuda.Stream(device, priority=hi), torch.cuda.Stream(device, priority=lo)
    ev = lambda: torch.cuda.Event(enable_timing=True)

    def time_fwd():
        with torch.cuda.stream(main):
            for _ in range(3):
                fwd_graph.replay()
        torch.cuda.synchronize()
        a, b = ev(), ev()
        a.record(main)
        with torch.cuda.stream(main):
            for _ in range(reps):
                fwd_graph.replay()
        b.record(main)
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps / 2 * 1e3            # us per layer

    dec_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(dec_graph, stream=side):
        for i in range(2):
            plans[i % 4].launch(side.cuda_stream)
    dec_graph2 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(dec_graph2, stream=side):
        for i in range(2, 4):
            plans[i].launch(side.cuda_stream)

    def time_dec():
        torch.cuda.synchronize()
        a, b = ev(), ev()
        a.record(side)
        with torch.cuda.stream(side):                      # replay() launches on the current stream
            for r in range(reps):
                (dec_graph if r % 2 == 0 else dec_graph2).replay()
        b.record(side)
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps / 2 * 1e3

    def time_both():
        torch.cuda.synchronize()
        a, b = ev(), ev()
        a.record(main)
        side.wait_event(a)
        for r in range(reps):
            with torch.cuda.stream(side):
                (dec_graph if r % 2 == 0 else dec_graph2).replay()
            with torch.cuda.stream(main):
                fwd_graph.replay()
        done = ev()
        done.record(side)
        main.wait_event(done)
        b.record(main)
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps / 2 * 1e3

    with torch.cuda.stream(side):                          # untimed first replays (graph upload)
        dec_graph.replay()
        dec_graph2.replay()
    torch.cuda.synchronize()
    t_fwd, t_dec = time_fwd(), time_dec()
    t_both = time_both()
    overlap = (t_dec + t_fwd - t_both) / min(t_dec, t_fwd)
    return {"workload": "config1 block: 2560/9728/32q/8kv/128, 7 RVQ projections (K=4, 256 codes, d=8, per-row "
                        "scales) decoded into a bf16 slot vs the batch-1 bf16 block forward (native decode step, "
                        "resident weights)",
            "t_fwd_us_per_layer": round(t_fwd, 2), "t_dec_us_per_layer": round(t_dec, 2),
            "t_both_us_per_layer": round(t_both, 2), "overlap": round(overlap, 3),
            "decode_GB/s_alone": round(algo / t_dec / 1e3, 1),
            "decode_added_us_per_layer_when_overlapped": round(t_both - t_fwd, 2),
            "decode_ctas": max_ctas or torch.cuda.get_device_properties(device).multi_processor_count,
            "forward_mode": forward_mode,
            "timing": "CUDA graphs replayed on two streams, CUDA events"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reps", type=int, default=50)
    ap.add_argument("--max-ctas", type=int, default=0)
    ap.add_argument("--forward", default="dense", choices=["dense", "fused"])
    a = ap.parse_args()
    print(json.dumps(run(a.reps, max_ctas=a.max_ctas, forward_mode=a.forward)))


if __name__ == "__main__":
    main()
