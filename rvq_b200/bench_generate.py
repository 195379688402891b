"""End-to-end batch-1 generation benchmark: random-init 36-layer Qwen3 model.

    python -m rvq_b200.bench_generate [--layers 36] [--prompt 128] [--new 128]

Model: the 2560 / 9728 / 32q / 8kv / head-128 block x 36 layers, vocab
151936, tied bf16 embeddings, RMSNorm, RoPE theta 1e6; every projection RVQ
(K=4, 256 codes, d=8, per-row fp16 scales).  The prompt is 128 ids drawn
uniformly from the vocab with a seed; 128 greedy new tokens.

Per weight mode of ``Qwen3Decoder`` (dense bf16 / slot decode + cuBLAS /
fused table GEMV / fused exact-weight GEMV) it reports TTFT (prefill + first argmax), ms/token (the
graph-replayed decode loop, device time by CUDA events, no host sync inside
the loop) and the generated ids; then it runs the reference's own engine
forward (``_layerwise_logits`` through HF modules on slot weights) for the
same prompt and checks the ids.  Prints one JSON object.
"""

from __future__ import annotations

import argparse
import json
import time

import torch

from . import synthetic
from .decoder import Qwen3Decoder
from .layerwise import (plan_from_module_tree, build_meta_model, generate_greedy_ids,
                        materialize_always_hot, upload_artifact)


def _events():
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def time_mode(dec: Qwen3Decoder, prompt: torch.Tensor, new: int, reps: int):
    dec.capture()
    dec.generate(prompt, 4)                       # warm-up: prefill kernels, graph upload
    torch.cuda.synchronize()
    ttft = []
    for _ in range(reps):
        s, e = _events()
        s.record()
        tok = dec.prefill(prompt).argmax()
        e.record()
        torch.cuda.synchronize()
        ttft.append(s.elapsed_time(e))
    # decode loop: the prefill is outside the timed region, every step inside
    logits = dec.prefill(prompt)
    tok = logits.argmax().view(1)
    toks = [tok]
    torch.cuda.synchronize()
    s, e = _events()
    s.record()
    pos = prompt.numel()
    for i in range(new - 1):
        tok = dec.step(tok, pos).argmax().view(1)
        toks.append(tok)
        pos += 1
    e.record()
    torch.cuda.synchronize()
    ms_tok = s.elapsed_time(e) / (new - 1)
    # the step alone (graph replays back to back)
    s, e = _events()
    s.record()
    for _ in range(20):
        dec.graph.replay()
    e.record()
    torch.cuda.synchronize()
    return {"ttft_ms": round(sorted(ttft)[len(ttft) // 2], 3), "ms_per_token": round(ms_tok, 4),
            "step_replay_ms": round(s.elapsed_time(e) / 20, 4)}, torch.cat(toks)


def margin(logits):
    top = torch.topk(logits.float().view(-1), 2).values
    return float(top[0] - top[1])


def run(layers=36, prompt_len=128, new=128, vocab=151936, reps=3,
        modes=("dense", "slot", "fused", "fused_exact", "fused_persistent"), reference=True, device="cuda:0", hbm_gbs=None):
    """TTFT, ms/token and greedy ids per weight mode, then the same prompt
    through the drop-in engine (``_layerwise_logits`` over HF decoder layers
    on slot weights, bit-identical to the oracle engine that is pinned to the
    reference engine's own output): per mode, whether the ids are identical,
    and if not the first divergence and the engine's top-1/top-2 margin there.
    ``hbm_gbs``: HBM peak for each mode's roofline fraction (weight bytes per
    token / ms per token)."""
    device = torch.device(device)
    torch.cuda.set_device(device)
    shape = synthetic.BlockShape()
    t0 = time.time()
    art = synthetic.make_tp_shard_artifact(shape, layers, vocab, 0, 1, seed=0, device=device)
    cfg = synthetic.qwen3_config(shape, layers, vocab)
    prompt = torch.randint(0, vocab, (prompt_len,), generator=torch.Generator().manual_seed(1234)).to(device)
    out = {"workload": f"Qwen3 block {shape.hidden}/{shape.intermediate}/{shape.n_heads}q/{shape.n_kv_heads}kv"
                       f"/{shape.head_dim} x {layers} layers, vocab {vocab}, tied bf16 embeddings, "
                       f"K=4 256-code d=8 RVQ with per-row scales, prompt {prompt_len}, {new} greedy tokens",
           "data": "synthetic random-init weights (generated on the GPU, seeded) and seeded prompt ids",
           "artifact_build_s": round(time.time() - t0, 1), "modes": {}}
    per_layer = shape.weights_per_block()
    head = vocab * shape.hidden * 2
    fused_bytes = layers * (per_layer // 8 * 4 + sum(o for _, o, _ in shape.projections()) * 2) + head
    bytes_tok = {"dense": layers * per_layer * 2 + head, "fused": fused_bytes, "fused_exact": fused_bytes,
                 "fused_persistent": fused_bytes}
    ids = {}
    for mode in modes:
        # "fused_persistent": fused weights, the whole step as one cooperative launch
        wmode, impl = ("fused", "persistent") if mode == "fused_persistent" else (mode, "native")
        dec = Qwen3Decoder(cfg, art, device, mode=wmode, max_len=prompt_len + new + 8, artifact_is_shard=True,
                           step_impl=impl)
        res, ids[mode] = time_mode(dec, prompt, new, reps)
        dec.check_waits()
        if mode in bytes_tok:
            res["weight_bytes_per_token"] = bytes_tok[mode]
            res["GB/s"] = round(bytes_tok[mode] / (res["ms_per_token"] * 1e6), 1)
            if hbm_gbs:
                res["roofline_frac"] = round(res["GB/s"] / hbm_gbs, 4)
        out["modes"][mode] = res
        del dec
        torch.cuda.empty_cache()
    if reference:
        model = build_meta_model(cfg)
        cbs, entries = upload_artifact(art, device)
        plan = plan_from_module_tree(model, entries)
        embed, lm_head = materialize_always_hot(model, plan, cbs, device, torch.bfloat16)
        torch.cuda.synchronize()
        t = time.time()
        ref_ids, ref_logits = generate_greedy_ids(model, plan, cbs, embed, lm_head, prompt.view(1, -1), new,
                                                  device, torch.bfloat16)
        torch.cuda.synchronize()
        ref_ids = ref_ids.view(-1)            # ref_logits[i] chose ref_ids[i]
        out["reference_engine"] = {
            "what": "the drop-in engine forward (_layerwise_logits through HF decoder layers, eager attention, "
                    "ping-pong slots), bit-identical to the oracle engine pinned to the reference engine's output",
            "ms_per_token_wall": round((time.time() - t) * 1e3 / (new + 1), 2),
            "min_top2_margin": round(min(margin(l) for l in ref_logits[:new]), 5)}
        for mode, got in ids.items():
            first = next((i for i in range(new) if int(got[i]) != int(ref_ids[i])), None)
            out["modes"][mode].update({
                "ids_identical_to_reference_engine": first is None, "first_divergence": first,
                "ref_margin_there": None if first is None else round(margin(ref_logits[first]), 5)})
        del model, plan, entries, embed, lm_head
    del art
    torch.cuda.empty_cache()
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=36)
    ap.add_argument("--prompt", type=int, default=128)
    ap.add_argument("--new", type=int, default=128)
    ap.add_argument("--vocab", type=int, default=151936)
    ap.add_argument("--modes", default="dense,slot,fused,fused_exact,fused_persistent")
    ap.add_argument("--no-reference", action="store_true")
    a = ap.parse_args(argv)
    print(json.dumps(run(a.layers, a.prompt, a.new, a.vocab, modes=tuple(a.modes.split(",")),
                         reference=not a.no_reference)))


if __name__ == "__main__":
    main()
