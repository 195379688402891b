"""Per-kernel timing of the fused batch-1 decode step, and small drivers for
profiling it.

    python -m rvq_b200.bench_step kernels --block config4 --layers 8
    python -m rvq_b200.bench_step one-step --block config4 --layers 2
    python -m rvq_b200.bench_step generate --block config1 --layers 4 --new 24

``kernels``: a random-init model of the block (vocab 151936, K=4 256-code
d=8 RVQ projections, per-row scales), 128-token prompt, then each kernel of
the native decode step (norm, q/k/v GEMV, attention, o GEMV, norm, gate+up
GEMV, down GEMV) replayed alone from a CUDA graph over all layers at
position 130; prints us per layer for each, the final norm + head, and the
whole step (CUDA events).  ``one-step``: prefill 16 ids and one eager decode
step (the launches an ncu capture selects from).  ``generate``: greedy
generation replaying the captured step.  The config-1 block is 2560 / 9728 /
32q / 8kv / 128, the config-4 block 5120 / 25600 / 64q / 8kv / 128.  With
``--tp N`` the kernels are timed on one rank's share of a TP=N model (heads,
kv heads and intermediate divided by N; no reduction).  ``--persistent``:
the decoder also holds the persistent step (rvq_b200/persist.py); ``kernels``
then times its one cooperative launch for all layers as well, and
``one-step`` runs it instead of the native step.
"""

from __future__ import annotations

import argparse
import json

import torch

from . import synthetic
from .decoder import Qwen3Decoder

BLOCKS = {
    "config1": synthetic.BlockShape(),
    "config4": synthetic.BlockShape(hidden=5120, intermediate=25600, n_heads=64, n_kv_heads=8, head_dim=128),
}


def rank_shape(block: str, tp: int) -> synthetic.BlockShape:
    """One tensor-parallel rank's share of the block: heads, kv heads and the
    intermediate size divided by tp (the shapes each GPU runs at TP = tp)."""
    b = BLOCKS[block]
    return synthetic.BlockShape(hidden=b.hidden, intermediate=b.intermediate // tp, n_heads=b.n_heads // tp,
                                n_kv_heads=b.n_kv_heads // tp, head_dim=b.head_dim)


def build(block: str, layers: int, vocab: int, max_len: int, device, tp: int = 1,
          persistent: bool = False) -> Qwen3Decoder:
    shape = rank_shape(block, tp)
    cfg = synthetic.qwen3_config(shape, layers, vocab)
    art = synthetic.make_tp_shard_artifact(shape, layers, vocab, 0, 1, seed=0, device=device)
    return Qwen3Decoder(cfg, art, device, mode="fused", max_len=max_len,
                        step_impl="persistent" if persistent else "native")


def time_kernels(block: str, layers: int, device, tp: int = 1, persistent: bool = False) -> dict:
    dec = build(block, layers, 151936, 256, device, tp, persistent)
    prompt = torch.randint(0, 151936, (128,), generator=torch.Generator().manual_seed(1)).to(device)
    dec.generate(prompt, 4)
    dec._pos.fill_(130)
    torch.cuda.synchronize()

    def graph_us(fn, reps=20):
        s = torch.cuda.Stream(device)
        s.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(s):
            fn()
        torch.cuda.current_stream(device).wait_stream(s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            g.replay()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps * 1e3

    res = {}
    for name in ("norm1", "qkv", "attn", "o", "norm2", "gu", "down"):
        def run(name=name):
            for l in range(layers):
                # layer 0's first norm embeds the token; time layer 1's in its place
                dec.step_ops[1 if (name == "norm1" and l == 0) else l][name].launch()
        res[name] = round(graph_us(run) / layers, 2)
    res["final_norm+head_per_token"] = round(graph_us(
        lambda: (dec.final_op.launch(), dec._mv(dec.lm_head, dec.x_final, dec.logits_buf))), 2)
    res["step_per_layer_incl_head"] = round(graph_us(dec._step_native) / layers, 2)
    if persistent:
        res["persistent_launch_per_layer"] = round(graph_us(dec.persist.launch) / layers, 2)
        res["persistent_step_per_layer_incl_head"] = round(graph_us(dec._step_persistent) / layers, 2)
        if dec.persist.take_error():
            raise RuntimeError("a persistent-step wait gave up during the timing")
    dec.close()
    return {"block": block, "tp_rank_share": tp, "layers": layers, "us_per_layer": res,
            "timing": "each kernel replayed alone from a CUDA graph over all layers, CUDA events"}


def one_step(block: str, layers: int, device, persistent: bool = False) -> None:
    dec = build(block, layers, 4096, 64, device, persistent=persistent)
    prompt = torch.randint(0, 4096, (16,), generator=torch.Generator().manual_seed(1)).to(device)
    with torch.inference_mode():
        dec.prefill(prompt)
        dec._tok.fill_(3)
        dec._pos.fill_(16)
        (dec._step_persistent if persistent else dec._step_native)()
    torch.cuda.synchronize()
    if persistent and dec.persist.take_error():
        raise RuntimeError("a persistent-step wait gave up")


def generate(block: str, layers: int, new: int, device) -> list:
    dec = build(block, layers, 151936, max(64, 16 + new + 8), device)
    prompt = torch.randint(0, 151936, (16,), generator=torch.Generator().manual_seed(1)).to(device)
    ids = dec.generate(prompt, new)
    torch.cuda.synchronize()
    return ids.tolist()


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=("kernels", "one-step", "generate"))
    ap.add_argument("--block", choices=tuple(BLOCKS), default="config1")
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--new", type=int, default=24)
    ap.add_argument("--tp", type=int, default=1, help="time one rank's share of a TP=tp model (kernels only)")
    ap.add_argument("--persistent", action="store_true", help="also time / run the persistent step")
    a = ap.parse_args(argv)
    device = torch.device("cuda:0")
    torch.cuda.set_device(device)
    if a.what == "kernels":
        print(json.dumps(time_kernels(a.block, a.layers, device, a.tp, a.persistent)))
    elif a.what == "one-step":
        one_step(a.block, a.layers, device, a.persistent)
        print("ok")
    else:
        print(json.dumps({"ids": generate(a.block, a.layers, a.new, device)}))


if __name__ == "__main__":
    main()
