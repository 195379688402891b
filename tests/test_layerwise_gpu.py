"""GPU: the drop-in layerwise engine and its ping-pong slots."""

import numpy as np
import pytest
import torch

from oracle.engine_ref import OracleEngine, oracle_weight
from rvq_b200 import synthetic
from rvq_b200.layerwise import (_layerwise_logits, plan_from_module_tree, build_meta_model,
                                generate_greedy_ids, materialize_always_hot, slots_for,
                                upload_artifact)

pytestmark = pytest.mark.gpu

TINY = synthetic.BlockShape(hidden=64, intermediate=128, n_heads=4, n_kv_heads=2, head_dim=16)
MID = synthetic.BlockShape(hidden=512, intermediate=1536, n_heads=8, n_kv_heads=2, head_dim=64)


def build_engine(shape, n_layers, vocab, seed, device, dtype=torch.bfloat16):
    art = synthetic.make_model_artifact(shape, n_layers, vocab, seed=seed)
    cfg = synthetic.qwen3_config(shape, n_layers, vocab)
    model = build_meta_model(cfg)
    gpu_codebooks, gpu_entries = upload_artifact(art, device)
    plan = plan_from_module_tree(model, gpu_entries)
    embed, lm_head = materialize_always_hot(model, plan, gpu_codebooks, device, dtype)
    return art, cfg, model, plan, gpu_codebooks, embed, lm_head


@pytest.mark.parametrize("shape,n_layers,vocab,seed,new_tokens", [
    (TINY, 2, 512, 5, 6),
    (TINY, 5, 512, 6, 8),          # odd layer count: slot of layer 0 alternates with the head
    (MID, 4, 4096, 7, 8),
])
def test_layerwise_matches_oracle_engine(shape, n_layers, vocab, seed, new_tokens, cuda_device):
    art, cfg, model, plan, cbs, embed, lm_head = build_engine(shape, n_layers, vocab, seed, cuda_device)
    g = torch.Generator().manual_seed(seed + 1)
    prompt = torch.randint(0, vocab, (1, 12), generator=g).to(cuda_device)
    ids, logits = generate_greedy_ids(model, plan, cbs, embed, lm_head, prompt, new_tokens,
                                      cuda_device, torch.bfloat16)
    ref = OracleEngine(synthetic.qwen3_config(shape, n_layers, vocab), art, cuda_device, torch.bfloat16)
    ref_ids, ref_logits = ref.generate(prompt, new_tokens)
    assert torch.equal(ids, ref_ids)
    for a, b in zip(logits, ref_logits):
        assert torch.equal(a, b)
    slots = slots_for(plan, cbs, cuda_device, torch.bfloat16)
    assert slots.launches == (n_layers * (new_tokens + 1) + 1)   # one launch per layer per pass + next-call prefetch


def test_slot_arena_is_reused_across_calls(cuda_device):
    art, cfg, model, plan, cbs, embed, lm_head = build_engine(TINY, 3, 512, 9, cuda_device)
    prompt = torch.randint(0, 512, (1, 5), generator=torch.Generator().manual_seed(1)).to(cuda_device)
    generate_greedy_ids(model, plan, cbs, embed, lm_head, prompt, 2, cuda_device, torch.bfloat16)
    slots = slots_for(plan, cbs, cuda_device, torch.bfloat16)
    ptrs = [b.data_ptr() for b in slots.arena.buffers]
    generate_greedy_ids(model, plan, cbs, embed, lm_head, prompt, 2, cuda_device, torch.bfloat16)
    assert slots_for(plan, cbs, cuda_device, torch.bfloat16) is slots
    assert [b.data_ptr() for b in slots.arena.buffers] == ptrs
    per_layer = sum(int(np.prod(e["shape"])) * 2 for k, e in plan["entries"].items()
                    if k.startswith("model.layers.0."))
    assert per_layer <= slots.slot_bytes < per_layer + 256 * 11


def test_slow_consumer_sees_its_own_layer(cuda_device):
    """The forward of layer l reads its slot for a long time (many matmuls)
    while layer l+1 (and l+2 into the same slot) are being decoded: every
    result must still equal the oracle's (refills wait for the free event)."""
    shape = synthetic.BlockShape(hidden=1024, intermediate=2048, n_heads=8, n_kv_heads=4, head_dim=128)
    n_layers = 6
    art = synthetic.make_model_artifact(shape, n_layers, 256, seed=11)
    cfg = synthetic.qwen3_config(shape, n_layers, 256)
    model = build_meta_model(cfg)
    cbs, entries = upload_artifact(art, cuda_device)
    plan = plan_from_module_tree(model, entries)
    slots = slots_for(plan, cbs, cuda_device, torch.bfloat16)
    x = torch.randn(64, shape.hidden, generator=torch.Generator().manual_seed(2)).to(cuda_device, torch.bfloat16)
    main = torch.cuda.current_stream()
    outs = []
    slots.prefetch(0)
    for l in range(n_layers):
        w = slots.acquire(l, main)
        slots.prefetch(l + 1)
        wq = w["self_attn.q_proj.weight"]
        acc = torch.zeros(64, wq.shape[0], device=cuda_device, dtype=torch.float32)
        for _ in range(200):                          # slow consumer of the slot
            acc += (x @ wq.t()).float()
        outs.append(acc)
        slots.release(l, main)
    torch.cuda.synchronize()
    for l in range(n_layers):
        wq = oracle_weight(art["entries"][f"model.layers.{l}.self_attn.q_proj.weight"],
                           art["shared_codebooks"], torch.bfloat16, cuda_device)
        want = torch.zeros_like(outs[l])
        for _ in range(200):
            want += (x @ wq.t()).float()
        assert torch.equal(outs[l], want), l
