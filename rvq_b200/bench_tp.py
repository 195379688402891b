"""Tensor-parallel batch-1 generation benchmark: random-init 64-layer model.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N \\
        --master-addr 127.0.0.1 --master-port 29511 -m rvq_b200.bench_tp [--layers 64]

Model: hidden 5120, intermediate 25600, 64 query / 8 kv heads of 128, 64
layers, vocab 151936, tied bf16 embeddings, RoPE theta 1e6; every projection
RVQ (K=4, 256 codes, d=8, per-row fp16 scales).  q/k/v/gate/up are
column-parallel, o/down row-parallel; their outputs are summed over the
ranks inside the captured CUDA graph, by peer stores into landing buffers
("push", rvq_b200/tp.py) or by an NCCL all-reduce ("nccl"; ``--reduce``).  Each rank generates its own shard on its GPU
(rank-seeded projections, common-seeded codebooks, norms and embedding), so
the ranks' shards form one consistent model.  Prompt: 128 seeded ids;
128 greedy tokens.  Rank 0 prints one JSON object: TTFT, ms/token (device
time, max over ranks), and per-GPU decode GB/s (the code bytes each GPU
reads per token / ms per token).
"""

from __future__ import annotations

import argparse
import datetime
import gc
import json
import os

import torch
import torch.distributed as dist

from . import synthetic
from .decoder import Qwen3Decoder

SHAPE = synthetic.BlockShape(hidden=5120, intermediate=25600, n_heads=64, n_kv_heads=8, head_dim=128)


def _max_over_ranks(v: float, device) -> float:
    t = torch.tensor([v], dtype=torch.float64, device=device)
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def bytes_per_token(shape, layers, vocab, tp):
    """HBM bytes one rank reads per token in the fused modes: its shard of every
    layer's codes (4 B per 8 weights) and row scales, and the replicated bf16
    head (tied embedding)."""
    local = synthetic.BlockShape(hidden=shape.hidden, intermediate=shape.intermediate // tp,
                                 n_heads=shape.n_heads // tp, n_kv_heads=shape.n_kv_heads // tp,
                                 head_dim=shape.head_dim)
    per_layer = sum(o * i // 2 + o * 2 for _, o, i in local.projections())
    return layers * per_layer + vocab * shape.hidden * 2


def measure(shape, layers, vocab, mode, device, group=None, prompt_len=128, new=128, seed=0, tp_reduce="push"):
    """TTFT and ms/token (device time, max over the group's ranks) of greedy
    generation for the rank's shard of a random model of ``shape``."""
    world = dist.get_world_size(group) if group is not None else 1
    rank = dist.get_rank(group) if group is not None else 0
    cfg = synthetic.qwen3_config(shape, layers, vocab)
    art = synthetic.make_tp_shard_artifact(shape, layers, vocab, rank, world, seed=seed, device=device)
    prompt = torch.randint(0, vocab, (prompt_len,), generator=torch.Generator().manual_seed(1234)).to(device)
    wmode, impl = ("fused", "persistent") if mode == "fused_persistent" else (mode, "native")
    dec = Qwen3Decoder(cfg, art, device, mode=wmode, max_len=prompt_len + new + 8, tp_group=group,
                       artifact_is_shard=True, tp_reduce=tp_reduce, step_impl=impl)
    del art
    dec.capture()
    dec.generate(prompt, 4)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ttft = []
    for _ in range(3):
        s.record()
        dec.prefill(prompt).argmax()
        e.record()
        torch.cuda.synchronize()
        ttft.append(s.elapsed_time(e))
    tok = dec.prefill(prompt).argmax().view(1)
    toks = [tok]
    if world > 1:
        dist.barrier(group)
    torch.cuda.synchronize()
    s.record()
    pos = prompt_len
    for _ in range(new - 1):
        tok = dec.step(tok, pos).argmax().view(1)
        toks.append(tok)
        pos += 1
    e.record()
    torch.cuda.synchronize()
    # a bounded device wait that gave up on any rank invalidates every rank's numbers
    try:
        dec.check_waits()
        waits_ok = 1.0
    except RuntimeError:
        waits_ok = 0.0
    if _max_over_ranks(1.0 - waits_ok, device) > 0:
        dec.close()
        raise RuntimeError("a bounded device wait timed out during the timed generation")
    ms_tok = _max_over_ranks(s.elapsed_time(e) / (new - 1), device)
    ttft_ms = _max_over_ranks(sorted(ttft)[1], device)
    ids = torch.cat(toks)
    same = True
    if world > 1:
        ref = ids.clone()
        dist.broadcast(ref, 0, group=group)
        flag = torch.tensor([float(torch.equal(ref, ids))], device=device)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
        same = bool(flag.item() == 1.0)
    dec.close()                      # releases the graph (it may hold NCCL calls) and the landing buffers
    del dec
    gc.collect()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return {"ttft_ms": round(ttft_ms, 3), "ms_per_token": round(ms_tok, 4), "ranks_agree_on_ids": same}


def run(layers=64, prompt_len=128, new=128, vocab=151936, modes=("fused",), reduces=("push",)):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device(f"cuda:{local}")
    torch.cuda.set_device(device)
    if world > 1:
        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=180))
    group = dist.group.WORLD if world > 1 else None
    per_layer = SHAPE.weights_per_block() // world
    code_bytes = layers * (per_layer // 8 * 4)
    out = {"workload": f"Qwen3-style {SHAPE.hidden}/{SHAPE.intermediate}/{SHAPE.n_heads}q/{SHAPE.n_kv_heads}kv/"
                       f"{SHAPE.head_dim} x {layers} layers, vocab {vocab}, K=4 256-code d=8 RVQ, per-row scales, "
                       f"prompt {prompt_len}, {new} greedy tokens",
           "tp": world, "data": "synthetic random-init shards generated per rank, seeded", "modes": {}}
    for mode in modes:
        for reduce in (reduces if world > 1 else ("push",)):
            res = measure(SHAPE, layers, vocab, mode, device, group, prompt_len, new, tp_reduce=reduce)
            if mode == "fused":
                res["code_bytes_per_gpu_per_token"] = code_bytes
                res["per_gpu_decode_GB/s"] = round(code_bytes / (res["ms_per_token"] * 1e6), 1)
            if world > 1:
                res["reductions_per_token"] = 2 * layers
                res["tp_reduce"] = reduce
            out["modes"][mode if world == 1 or len(reduces) == 1 else f"{mode}+{reduce}"] = res
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=64)
    ap.add_argument("--prompt", type=int, default=128)
    ap.add_argument("--new", type=int, default=128)
    ap.add_argument("--vocab", type=int, default=151936)
    ap.add_argument("--modes", default="fused")
    ap.add_argument("--reduce", default="push", help="push, nccl or push,nccl")
    a = ap.parse_args(argv)
    res = run(a.layers, a.prompt, a.new, a.vocab, tuple(a.modes.split(",")), tuple(a.reduce.split(",")))
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps(res))
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
