"""GPU: the persistent decode step (rvq_persist_step, one cooperative launch
per token) against the plain native step (seven launches per layer) of the
same fused-mode decoder.

Every phase of the persistent kernel repeats the arithmetic of the kernel it
replaces in the same order, so logits, the residual stream and the KV cache
must be BIT-identical, step after step; greedy generation must give the same
ids.  The plain native step is itself pinned to the reference engine by
tests/test_decoder_gpu.py.
"""

import pytest
import torch

from rvq_b200 import _native, synthetic
from rvq_b200.decoder import Qwen3Decoder

pytestmark = pytest.mark.gpu

SHAPES = {
    "rep4": synthetic.BlockShape(hidden=1024, intermediate=2816, n_heads=8, n_kv_heads=2, head_dim=128),
    "rep8": synthetic.BlockShape(hidden=1024, intermediate=3072, n_heads=16, n_kv_heads=2, head_dim=128),
    "rep1_ragged": synthetic.BlockShape(hidden=640, intermediate=1000, n_heads=4, n_kv_heads=4, head_dim=128),
    "qwen_block": synthetic.BlockShape(),          # 2560 / 9728, 32 q / 8 kv heads
}


def run_pair(shape, layers, vocab, prompt_len, steps, max_len, seed, device, causal=False):
    art = synthetic.make_model_artifact(shape, layers, vocab, seed=seed)
    cfg = synthetic.qwen3_config(shape, layers, vocab)
    g = torch.Generator().manual_seed(seed + 1)
    prompt = torch.randint(0, vocab, (prompt_len,), generator=g).to(device)
    ids = torch.randint(0, vocab, (steps,), generator=g).to(device)
    out = []
    for impl in ("native", "persistent"):
        dec = Qwen3Decoder(cfg, art, device, mode="fused", max_len=max_len, causal=causal, step_impl=impl)
        logits = [dec.prefill(prompt).float().clone()]
        hs = []
        for i, t in enumerate(ids.tolist()):
            logits.append(dec.step(torch.tensor([t], device=device), prompt_len + i).float().clone())
            hs.append(dec.h.clone())
        dec.check_waits()
        out.append((logits, hs, dec.k_cache.clone(), dec.v_cache.clone()))
        dec.close()
        del dec
    return out


@pytest.mark.parametrize("name,layers,vocab,prompt_len,steps,max_len,causal", [
    ("rep4", 3, 4096, 20, 12, 64, False),
    ("rep4", 2, 4096, 20, 6, 64, True),
    ("rep8", 2, 4096, 9, 10, 48, False),
    ("rep1_ragged", 2, 2048, 5, 8, 32, False),
    ("rep4", 2, 4096, 300, 6, 320, False),         # 306 keys: 38-39 in each key range of the attention
    ("qwen_block", 2, 8192, 24, 8, 64, False),
])
def test_persistent_step_bit_identical_to_native(name, layers, vocab, prompt_len, steps, max_len, causal,
                                                 cuda_device):
    (ln, hn, kn, vn), (lp, hp, kp, vp) = run_pair(SHAPES[name], layers, vocab, prompt_len, steps, max_len,
                                                  seed=len(name) * 7 + layers, device=cuda_device,
                                                  causal=causal)
    assert torch.equal(ln[0], lp[0])               # the prompt: the same PyTorch ops
    for i in range(steps):
        assert torch.equal(hn[i], hp[i]), i
        assert torch.equal(ln[i + 1], lp[i + 1]), i
    assert torch.equal(kn, kp) and torch.equal(vn, vp)


def test_persistent_generate_matches_native(cuda_device):
    shape = SHAPES["rep4"]
    art = synthetic.make_model_artifact(shape, 3, 4096, seed=5)
    cfg = synthetic.qwen3_config(shape, 3, 4096)
    prompt = torch.randint(0, 4096, (16,), generator=torch.Generator().manual_seed(6)).to(cuda_device)
    res = []
    for impl in ("native", "persistent"):
        dec = Qwen3Decoder(cfg, art, cuda_device, mode="fused", max_len=64, step_impl=impl)
        ids, logits = dec.generate(prompt, 24, return_logits=True)
        ids2 = dec.generate(prompt, 24)             # a second run replays the same graph
        dec.check_waits()
        assert torch.equal(ids, ids2)
        res.append((ids, logits))
        dec.close()
    assert torch.equal(res[0][0], res[1][0])
    for a, b in zip(res[0][1], res[1][1]):
        assert torch.equal(a, b)


def test_persistent_wait_gives_up_and_next_step_recovers(cuda_device):
    """A phase counter that cannot reach its target (set far below it before
    the launch): every wait gives up after about a second, the step ends, the
    sticky flag reads 1 once, and the counters are back at zero, so the next
    step at the same position is exact again."""
    shape = SHAPES["rep4"]
    art = synthetic.make_model_artifact(shape, 2, 2048, seed=9)
    cfg = synthetic.qwen3_config(shape, 2, 2048)
    prompt = torch.randint(0, 2048, (8,), generator=torch.Generator().manual_seed(10)).to(cuda_device)
    ref = Qwen3Decoder(cfg, art, cuda_device, mode="fused", max_len=32)
    ref.prefill(prompt)
    want = ref.step(torch.tensor([7], device=cuda_device), 8).clone()
    ref.close()
    dec = Qwen3Decoder(cfg, art, cuda_device, mode="fused", max_len=32, step_impl="persistent")
    dec.prefill(prompt)
    assert not dec.persist.take_error()
    dec._tok.fill_(7)
    dec._pos.fill_(8)
    dec.persist.sync[0] = -(2 ** 31)              # the norm counter: never reaches 8
    dec.persist.launch()
    assert dec.persist.take_error()
    assert not dec.persist.take_error()             # read and cleared
    counters = [0, 32, 64] + [128 + 32 * k for k in range(16)]        # norm, attention, exit, GEMV
    assert int(dec.persist.sync[counters].abs().sum()) == 0
    got = dec.step(torch.tensor([7], device=cuda_device), 8)
    dec.check_waits()
    assert torch.equal(got, want)
    dec.close()


def test_persistent_rejects_what_it_cannot_run(cuda_device):
    mid = synthetic.BlockShape(hidden=512, intermediate=1536, n_heads=8, n_kv_heads=2, head_dim=64)
    art = synthetic.make_model_artifact(mid, 1, 1024, seed=3)
    cfg = synthetic.qwen3_config(mid, 1, 1024)
    with pytest.raises(_native.RvqError) as e:      # head_dim 64: the planner says unsupported
        Qwen3Decoder(cfg, art, cuda_device, mode="fused", max_len=32, step_impl="persistent")
    assert e.value.status == _native.RVQ_ERR_UNSUPPORTED
    with pytest.raises(NotImplementedError):
        Qwen3Decoder(cfg, art, cuda_device, mode="slot", max_len=32, step_impl="persistent")
    shape = SHAPES["rep8"]
    art = synthetic.make_model_artifact(shape, 1, 1024, seed=4)
    cfg = synthetic.qwen3_config(shape, 1, 1024)
    with pytest.raises(_native.RvqError) as e:      # 8 heads per kv head x 2048 rows > 15360 scores
        Qwen3Decoder(cfg, art, cuda_device, mode="fused", max_len=2048, step_impl="persistent")
    assert e.value.status == _native.RVQ_ERR_TOO_LARGE
