"""GPU: the decode-step kernels (rvq_step_norm / _attention / _silu_mul)
against the PyTorch ops of the HF Qwen3 modules they replace.

Rounding points are the same as HF's; only fp32 summation order differs, so
results agree to one bf16 ulp on a small fraction of elements at most.
"""

import pytest
import torch
import torch.nn.functional as F

from rvq_b200.decoder import rmsnorm, rotate_half
from rvq_b200.step import AttentionOp, NormOp, SiluMulOp

pytestmark = pytest.mark.gpu


def ulp_diff(a, b):
    """|a - b| in units of the bf16 ulp of the larger magnitude."""
    a, b = a.float(), b.float()
    m = torch.maximum(a.abs(), b.abs()).clamp_min(2.0 ** -126)
    ulp = torch.ldexp(torch.ones_like(m), torch.frexp(m).exponent - 8)
    return ((a - b).abs() / ulp).round().to(torch.int64)


def assert_close_ulp(got, want, max_ulp=1, max_frac=0.02):
    d = ulp_diff(got, want)
    assert int(d.max()) <= max_ulp, int(d.max())
    assert float((d > 0).float().mean()) <= max_frac, float((d > 0).float().mean())


@pytest.mark.parametrize("hidden,ntiles", [(2560, 1), (2560, 16), (5120, 38), (333, 3)])
def test_norm_matches_hf_rmsnorm(hidden, ntiles, cuda_device):
    g = torch.Generator().manual_seed(hidden + ntiles)
    h0 = torch.randn(hidden, generator=g).to(cuda_device, torch.bfloat16)
    w = (1 + 0.1 * torch.randn(hidden, generator=g)).to(cuda_device, torch.bfloat16)
    if ntiles == 1:
        add = torch.randn(hidden, generator=g).to(cuda_device, torch.bfloat16)
        add_val = add
    else:
        add = torch.randn(ntiles, hidden, generator=g).to(cuda_device) / ntiles
        s = add[0].clone()
        for t in range(1, ntiles):
            s += add[t]
        add_val = s.to(torch.bfloat16)
    h = h0.clone()
    x = torch.empty_like(h)
    NormOp(h, w, x, 1e-6, add=add, add_tiles=ntiles).launch()
    torch.cuda.synchronize()
    h_want = h0 + add_val
    assert torch.equal(h, h_want)
    assert_close_ulp(x, rmsnorm(h_want, w, 1e-6))


def test_norm_embeds_token(cuda_device):
    g = torch.Generator().manual_seed(7)
    embed = torch.randn(100, 2560, generator=g).to(cuda_device, torch.bfloat16)
    w = (1 + 0.1 * torch.randn(2560, generator=g)).to(cuda_device, torch.bfloat16)
    tok = torch.tensor([42], device=cuda_device)
    h = torch.zeros(2560, dtype=torch.bfloat16, device=cuda_device)
    x = torch.empty_like(h)
    NormOp(h, w, x, 1e-6, token=tok, embed=embed).launch()
    torch.cuda.synchronize()
    assert torch.equal(h, embed[42])
    assert_close_ulp(x, rmsnorm(embed[42], w, 1e-6))


def torch_attention(q, k, v, qn, kn, cos, sin, pos, kc, vc, nh, nkv, hd, eps, scaling, bias):
    """The decoder's PyTorch decode-step attention (static cache, masked)."""
    rep = nh // nkv
    q = rmsnorm(q.view(1, 1, nh, hd), qn, eps).transpose(1, 2)
    k = rmsnorm(k.view(1, 1, nkv, hd), kn, eps).transpose(1, 2)
    v = v.view(1, 1, nkv, hd).transpose(1, 2)
    c, s = cos[pos].view(1, 1, 1, hd), sin[pos].view(1, 1, 1, hd)
    q = q * c + rotate_half(q) * s
    k = k * c + rotate_half(k) * s
    kc[:, pos] = k[0, :, 0]
    vc[:, pos] = v[0, :, 0]
    L = pos + 1
    sc = torch.matmul(q.view(nkv, rep, hd), kc[:, :L].transpose(1, 2)) * scaling
    sc = sc + torch.tensor(bias, dtype=torch.bfloat16, device=q.device)
    p = torch.softmax(sc, dim=-1, dtype=torch.float32).to(torch.bfloat16)
    return torch.matmul(p, vc[:, :L]).reshape(-1)


@pytest.mark.parametrize("nh,nkv,hd,pos,bias,partials", [
    (32, 8, 128, 0, 1.0, False), (32, 8, 128, 127, 1.0, False), (32, 8, 128, 300, 0.0, True),
    (64, 8, 128, 200, 1.0, True), (8, 2, 64, 50, 1.0, False), (16, 16, 256, 17, 0.0, False)])
@pytest.mark.parametrize("short_cache", [False, True])
def test_attention_matches_torch(nh, nkv, hd, pos, bias, partials, short_cache, cuda_device):
    """A 512-row cache and one of pos + 40 rows (the keys split over the
    8-CTA cluster differ)."""
    g = torch.Generator().manual_seed(nh * 1000 + pos)
    max_len = pos + 40 if short_cache else 512
    dev = cuda_device
    bf = torch.bfloat16
    kc = (torch.randn(nkv, max_len, hd, generator=g)).to(dev, bf)
    vc = (torch.randn(nkv, max_len, hd, generator=g)).to(dev, bf)
    qn = (1 + 0.1 * torch.randn(hd, generator=g)).to(dev, bf)
    kn = (1 + 0.1 * torch.randn(hd, generator=g)).to(dev, bf)
    ang = torch.outer(torch.arange(max_len).float(), 1.0 / (1e6 ** (torch.arange(0, hd, 2).float() / hd)))
    emb = torch.cat([ang, ang], -1)
    cos, sin = emb.cos().to(dev, bf), emb.sin().to(dev, bf)
    if partials:
        qp = torch.randn(4, nh * hd, generator=g).to(dev) / 2
        kp = torch.randn(4, nkv * hd, generator=g).to(dev) / 2
        vp = torch.randn(4, nkv * hd, generator=g).to(dev) / 2
        red = lambda p: ((p[0] + p[1]) + p[2] + p[3]).to(bf)
        q, k, v, tiles = red(qp), red(kp), red(vp), 4
        ins = (qp, kp, vp)
    else:
        q = torch.randn(nh * hd, generator=g).to(dev, bf)
        k = torch.randn(nkv * hd, generator=g).to(dev, bf)
        v = torch.randn(nkv * hd, generator=g).to(dev, bf)
        tiles = 1
        ins = (q, k, v)
    kc2, vc2 = kc.clone(), vc.clone()
    want = torch_attention(q, k, v, qn, kn, cos, sin, pos, kc2, vc2, nh, nkv, hd, 1e-6, hd ** -0.5, bias)
    out = torch.empty(nh * hd, dtype=bf, device=dev)
    p = torch.tensor([pos], device=dev)
    AttentionOp(*ins, qn, kn, cos, sin, p, kc, vc, out, n_heads=nh, n_kv=nkv, head_dim=hd, eps=1e-6,
                scaling=hd ** -0.5, valid_bias=bias, q_tiles=tiles, kv_tiles=tiles).launch()
    torch.cuda.synchronize()
    others = torch.ones(max_len, dtype=torch.bool, device=dev)
    others[pos] = False
    assert torch.equal(kc[:, others], kc2[:, others]) and torch.equal(vc, vc2)   # only row pos written
    assert_close_ulp(kc[:, pos], kc2[:, pos], max_ulp=1, max_frac=0.05)
    rel = float((out.float() - want.float()).norm() / want.float().norm())
    assert rel < 4e-3, rel
    # a weighted sum of signed values: near-zero outputs make ulps meaningless,
    # so bound the absolute difference by the output's rms, and count ulp misses
    rms = float(want.float().pow(2).mean().sqrt())
    assert float((out.float() - want.float()).abs().max()) <= 0.02 * rms
    assert float((ulp_diff(out, want) > 1).float().mean()) <= 0.01


@pytest.mark.parametrize("n,tiles", [(9728, 1), (9728, 10), (25600, 38)])
def test_silu_mul_matches_torch(n, tiles, cuda_device):
    g = torch.Generator().manual_seed(n + tiles)
    if tiles == 1:
        gate = (3 * torch.randn(n, generator=g)).to(cuda_device, torch.bfloat16)
        up = torch.randn(n, generator=g).to(cuda_device, torch.bfloat16)
        gv, uv = gate, up
    else:
        gate = torch.randn(tiles, n, generator=g).to(cuda_device)
        up = torch.randn(tiles, n, generator=g).to(cuda_device)
        def red(p):
            s = p[0].clone()
            for t in range(1, tiles):
                s += p[t]
            return s.to(torch.bfloat16)
        gv, uv = red(gate), red(up)
    out = torch.empty(n, dtype=torch.bfloat16, device=cuda_device)
    SiluMulOp(gate, up, out, tiles, tiles).launch()
    torch.cuda.synchronize()
    assert_close_ulp(out, F.silu(gv) * uv, max_ulp=1, max_frac=0.01)
