"""CPU: the decoder's norm and rotary math equal the HF Qwen3 modules bit for bit."""

import torch

from rvq_b200 import synthetic
from rvq_b200.decoder import Dims, rmsnorm, rotate_half


def test_rmsnorm_equals_hf_module():
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RMSNorm
    g = torch.Generator().manual_seed(0)
    m = Qwen3RMSNorm(256, eps=1e-6)
    with torch.no_grad():
        m.weight.copy_(1 + 0.02 * torch.randn(256, generator=g))
    m = m.to(torch.bfloat16)
    x = torch.randn(5, 256, generator=g).to(torch.bfloat16)
    assert torch.equal(rmsnorm(x, m.weight, 1e-6), m(x))


def test_rotary_equals_hf_module():
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RotaryEmbedding, apply_rotary_pos_emb
    shape = synthetic.BlockShape(hidden=256, intermediate=512, n_heads=4, n_kv_heads=2, head_dim=64)
    cfg = synthetic.qwen3_config(shape, 2, 128)
    d = Dims.from_config(cfg)
    assert d.theta == 1e6
    rot = Qwen3RotaryEmbedding(cfg)
    T = 37
    x = torch.randn(1, T, d.hidden).to(torch.bfloat16)
    cos_hf, sin_hf = rot(x, torch.arange(T).unsqueeze(0))
    inv = 1.0 / (d.theta ** (torch.arange(0, d.head_dim, 2, dtype=torch.int64).float() / d.head_dim))
    emb = torch.cat([torch.outer(torch.arange(T).float(), inv)] * 2, dim=-1)
    assert torch.equal(emb.cos().to(torch.bfloat16), cos_hf[0])
    assert torch.equal(emb.sin().to(torch.bfloat16), sin_hf[0])
    q = torch.randn(1, d.n_heads, T, d.head_dim).to(torch.bfloat16)
    k = torch.randn(1, d.n_kv, T, d.head_dim).to(torch.bfloat16)
    qh, kh = apply_rotary_pos_emb(q, k, cos_hf, sin_hf)
    c, s = cos_hf[0], sin_hf[0]
    assert torch.equal(q * c + rotate_half(q) * s, qh)
    assert torch.equal(k * c + rotate_half(k) * s, kh)
