"""GPU: rvq_gemv_tiles (per-tile partial sums) against the oracle's reconstruction.

Each tile's partial sum is compared with the fp64 product of the oracle's
fp32 weight restricted to that tile's 256 columns.  The tables hold fp16
entries of codeword . (2^-E x) (one rounding, relative error <= 2^-11 per
entry, random in sign), so the sums agree to ~1.5e-4 relative; the bound
here is TOL = 1e-3, still 4x below the 2^-9 relative rounding of a bf16 weight
that the reference's reconstruct-then-matmul incurs.
"""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle.rvq_oracle import OUT_F32, RVQEntryNP, decode_rvq
from rvq_b200 import synthetic
from rvq_b200.gemv import GemvTilesPlan, tile_codes, tiles_count

pytestmark = pytest.mark.gpu

TOL = 1e-3


def oracle_w(entry, cb):
    numel = int(np.prod(entry["shape"]))
    e = RVQEntryNP(indices=entry["indices"].numpy(), codebook=cb.float().numpy(),
                   scales=entry["scales"].float().numpy(), tail=entry["tail"].float().numpy(), d=8,
                   group_size=int(entry["group_size"]), trimmed_numel=int(entry["trimmed_numel"]),
                   numel=numel)
    return decode_rvq(e, OUT_F32).reshape(entry["shape"]).astype(np.float64)


def dev_entry(entry, device):
    e = {k: (v.to(device) if torch.is_tensor(v) else v) for k, v in entry.items()}
    rows, cols = (int(v) for v in e["shape"])
    e["codes_tiled"] = tile_codes(e["indices"], rows, cols)
    return e


def rel_err(got, want):
    got = np.asarray(got, np.float64)
    return float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30))


def tile_products(w, x):
    cols = w.shape[1]
    return np.stack([w[:, t * 256:(t + 1) * 256] @ x[t * 256:(t + 1) * 256] for t in range(tiles_count(cols))])


@pytest.mark.parametrize("rows,cols,group,cb_dtype", [
    (9728, 2560, None, torch.float32),     # gate projection, per-row scales
    (2560, 9728, None, torch.float32),     # down projection, 38 tiles
    (4096, 2560, None, torch.float16),     # fp16 codebook
    (1024, 2560, 128, torch.float32),      # 16 vectors per scale
    (333, 520, None, torch.float32),       # ragged last tile (1 group), odd rows
    (8, 8, 8, torch.float32),              # one vector per row
    (3000, 1000, 40, torch.float32),       # G = 125: rows not 16-byte aligned, 5 vectors per scale
    (2048, 2560, None, "f32_not_f16"),     # fp32 codebook that fp16 cannot hold: fp32 staging
])
def test_tiles_match_reconstruction(rows, cols, group, cb_dtype, cuda_device):
    g = torch.Generator().manual_seed(rows + 3 * cols)
    cb = synthetic.make_codebook(4, 256, 8, g)
    if cb_dtype == "f32_not_f16":
        cb = cb.float() * (1 + 1e-6 * torch.randn(cb.shape, generator=g))
        assert not torch.equal(cb.half().float(), cb)
        cb_dtype = torch.float32
    entry = synthetic.make_rvq_entry(rows, cols, g, group_size=group)
    x = torch.randn(cols, generator=g).to(torch.bfloat16)
    part = torch.full((tiles_count(cols), rows), float("nan"), device=cuda_device)
    GemvTilesPlan([(dev_entry(entry, cuda_device), cb.to(cuda_device, cb_dtype), x.to(cuda_device), part)]).launch()
    torch.cuda.synchronize()
    assert not torch.isnan(part).any()
    w = oracle_w(entry, cb)
    xd = x.double().numpy()
    tp = tile_products(w, xd)
    assert rel_err(part.cpu().numpy(), tp) <= TOL
    assert rel_err(part.sum(0).cpu().numpy(), w @ xd) <= TOL


def test_multi_job_launch_and_determinism(cuda_device):
    """q, k, v in one launch (different codebooks, shared x); repeated
    launches give bit-identical partials."""
    g = torch.Generator().manual_seed(11)
    shapes = [(4096, 2560), (1024, 2560), (1024, 2560)]
    cbs = [synthetic.make_codebook(4, 256, 8, g) for _ in shapes]
    entries = [synthetic.make_rvq_entry(r, c, g) for r, c in shapes]
    x = torch.randn(2560, generator=g).to(torch.bfloat16)
    xd = x.to(cuda_device)
    parts = [torch.zeros(tiles_count(c), r, device=cuda_device) for r, c in shapes]
    plan = GemvTilesPlan([(dev_entry(e, cuda_device), cb.to(cuda_device, torch.float32), xd, p)
                          for e, cb, p in zip(entries, cbs, parts)])
    plan.launch()
    torch.cuda.synchronize()
    first = [p.clone() for p in parts]
    for _ in range(3):
        plan.launch()
    torch.cuda.synchronize()
    for e, cb, p, p0 in zip(entries, cbs, parts, first):
        assert torch.equal(p, p0)
        assert rel_err(p.cpu().numpy(), tile_products(oracle_w(e, cb), x.double().numpy())) <= TOL


def test_partial_operand_and_fused_silu(cuda_device):
    """The down projection's input straight from the gate / up partials:
    operand = bf16(bf16(silu(gate)) * up), each the tile-ordered sum of its
    partials rounded to bf16."""
    g = torch.Generator().manual_seed(12)
    rows, cols, nt = 2560, 9728, 10
    cb = synthetic.make_codebook(4, 256, 8, g)
    entry = synthetic.make_rvq_entry(rows, cols, g)
    gate_p = (torch.randn(nt, cols, generator=g) / 3).to(cuda_device)
    up_p = (torch.randn(nt, cols, generator=g) / 3).to(cuda_device)

    def tile_sum(p):
        s = p[0].clone()
        for t in range(1, nt):
            s += p[t]
        return s.to(torch.bfloat16)

    act = (F.silu(tile_sum(gate_p)) * tile_sum(up_p)).double().cpu().numpy()
    part = torch.zeros(tiles_count(cols), rows, device=cuda_device)
    GemvTilesPlan([(dev_entry(entry, cuda_device), cb.to(cuda_device, torch.float32), up_p, part, gate_p)]).launch()
    torch.cuda.synchronize()
    w = oracle_w(entry, cb)
    assert rel_err(part.sum(0).cpu().numpy(), w @ act) <= TOL
    # the same with the plain operand (no gate): x = up partials
    part2 = torch.zeros_like(part)
    GemvTilesPlan([(dev_entry(entry, cuda_device), cb.to(cuda_device, torch.float32), up_p, part2)]).launch()
    torch.cuda.synchronize()
    assert rel_err(part2.sum(0).cpu().numpy(), w @ tile_sum(up_p).double().cpu().numpy()) <= TOL


def test_tile_codes_layout(cuda_device):
    """rvq_tile_codes against a host restatement of the layout: word (t, r, w)
    = the stage codes of vector (r, 32 t + w), stage k in byte k, zero past
    the last group of a row."""
    g = torch.Generator().manual_seed(14)
    for rows, cols in [(5, 264), (40, 2560), (3, 8)]:
        entry = synthetic.make_rvq_entry(rows, cols, g)
        planes = entry["indices"].numpy().astype(np.uint32)
        G, nt = cols // 8, tiles_count(cols)
        words = planes[0] | (planes[1] << 8) | (planes[2] << 16) | (planes[3] << 24)
        want = np.zeros((nt, rows, 32), np.uint32)
        for t in range(nt):
            gs = min(32, G - 32 * t)
            want[t, :, :gs] = words.reshape(rows, G)[:, 32 * t:32 * t + gs]
        got = tile_codes(entry["indices"].to(cuda_device), rows, cols).cpu().numpy().view(np.uint32)
        assert np.array_equal(got.reshape(nt, rows, 32), want)


def test_rejects_bad_jobs(cuda_device):
    g = torch.Generator().manual_seed(13)
    cb = synthetic.make_codebook(4, 256, 8, g).to(cuda_device, torch.float32)
    e = dev_entry(synthetic.make_rvq_entry(64, 256, g), cuda_device)
    x = torch.zeros(256, dtype=torch.bfloat16, device=cuda_device)
    with pytest.raises(ValueError):
        GemvTilesPlan([(e, cb, x, torch.zeros(2, 64, device=cuda_device))])        # wrong tile count
    with pytest.raises(ValueError):
        GemvTilesPlan([(e, cb, torch.zeros(128, dtype=torch.bfloat16, device=cuda_device),
                        torch.zeros(1, 64, device=cuda_device))])                     # wrong operand length


# ---------------------------------------------------------------------------
# rvq_gemv_tiles_exact: bit-exact bf16 weights, fp32 products
# ---------------------------------------------------------------------------

# fp32 summation of at most 256 exact bf16 x bf16 products per tile
TOL_EXACT = 2e-6


def oracle_w_bf16(entry, cb):
    """The decoded slot's bf16 weights (the reference's reconstruction, RNE), as fp64."""
    from oracle.rvq_oracle import OUT_BF16, bf16_bits_to_f32, decode_rvq_bits
    numel = int(np.prod(entry["shape"]))
    e = RVQEntryNP(indices=entry["indices"].numpy(), codebook=cb.float().numpy(),
                   scales=entry["scales"].float().numpy(), tail=entry["tail"].float().numpy(), d=8,
                   group_size=int(entry["group_size"]), trimmed_numel=int(entry["trimmed_numel"]),
                   numel=numel)
    return bf16_bits_to_f32(decode_rvq_bits(e, OUT_BF16)).reshape(entry["shape"]).astype(np.float64)


@pytest.mark.parametrize("rows,cols,group,cb_dtype", [
    (9728, 2560, None, torch.float32),     # gate projection, per-row scales, fp32 codebook (fp16 values)
    (2560, 9728, None, torch.float16),     # down projection, 38 tiles, fp16 codebook
    (1024, 2560, 128, torch.float32),      # 16 vectors per scale
    (333, 520, None, torch.float32),       # ragged last tile (1 group), odd rows
    (8, 8, 8, torch.float32),              # one vector per row
    (3000, 1000, 40, torch.float32),       # 5 vectors per scale, scales change inside a tile row
    (2048, 2560, None, "f32_not_f16"),     # fp32 codebook that fp16 cannot hold: global fp32 path
])
def test_exact_tiles_match_bf16_weights(rows, cols, group, cb_dtype, cuda_device):
    g = torch.Generator().manual_seed(rows + 5 * cols)
    cb = synthetic.make_codebook(4, 256, 8, g)
    if cb_dtype == "f32_not_f16":
        cb = cb.float() * (1 + 1e-6 * torch.randn(cb.shape, generator=g))
        assert not torch.equal(cb.half().float(), cb)
        cb_dtype = torch.float32
    entry = synthetic.make_rvq_entry(rows, cols, g, group_size=group)
    x = torch.randn(cols, generator=g).to(torch.bfloat16)
    part = torch.full((tiles_count(cols), rows), float("nan"), device=cuda_device)
    GemvTilesPlan([(dev_entry(entry, cuda_device), cb.to(cuda_device, cb_dtype), x.to(cuda_device), part)],
                  exact=True).launch()
    torch.cuda.synchronize()
    assert not torch.isnan(part).any()
    w = oracle_w_bf16(entry, cb)
    xd = x.double().numpy()
    assert rel_err(part.cpu().numpy(), tile_products(w, xd)) <= TOL_EXACT
    got = part.sum(0).cpu().double().numpy()
    assert rel_err(got, w @ xd) <= TOL_EXACT
    # F.linear on the decoded bf16 slot (cuBLAS): the same products, another summation order
    slot = torch.from_numpy(w).to(torch.bfloat16).to(cuda_device)
    lin = F.linear(x.to(cuda_device).float().view(1, -1), slot.float()).view(-1).double().cpu().numpy()
    assert rel_err(got, lin) <= 1e-5


def test_exact_partial_operand_fused_silu_and_determinism(cuda_device):
    g = torch.Generator().manual_seed(22)
    rows, cols, nt = 2560, 9728, 10
    cb = synthetic.make_codebook(4, 256, 8, g)
    entry = dev_entry(synthetic.make_rvq_entry(rows, cols, g), cuda_device)
    gate_p = (torch.randn(nt, cols, generator=g) / 3).to(cuda_device)
    up_p = (torch.randn(nt, cols, generator=g) / 3).to(cuda_device)

    def tile_sum(p):
        s = p[0].clone()
        for t in range(1, nt):
            s += p[t]
        return s.to(torch.bfloat16)

    act = (F.silu(tile_sum(gate_p)) * tile_sum(up_p)).double().cpu().numpy()
    part = torch.zeros(tiles_count(cols), rows, device=cuda_device)
    plan = GemvTilesPlan([(entry, cb.to(cuda_device, torch.float32), up_p, part, gate_p)], exact=True)
    plan.launch()
    torch.cuda.synchronize()
    first = part.clone()
    host_entry = {k: (v.cpu() if torch.is_tensor(v) else v) for k, v in entry.items()}
    w = oracle_w_bf16(host_entry, cb)
    assert rel_err(part.sum(0).cpu().numpy(), w @ act) <= TOL_EXACT
    for _ in range(3):
        plan.launch()
    torch.cuda.synchronize()
    assert torch.equal(part, first)
    from rvq_b200.gemv import take_wait_timeout
    assert not take_wait_timeout()


def test_exact_rejects_fp16_operand(cuda_device):
    from rvq_b200 import _native
    g = torch.Generator().manual_seed(23)
    cb = synthetic.make_codebook(4, 256, 8, g).to(cuda_device, torch.float32)
    e = dev_entry(synthetic.make_rvq_entry(64, 256, g), cuda_device)
    x = torch.zeros(256, dtype=torch.float16, device=cuda_device)
    plan = GemvTilesPlan([(e, cb, x, torch.zeros(1, 64, device=cuda_device))], exact=True)
    with pytest.raises(_native.RvqError):
        plan.launch()
