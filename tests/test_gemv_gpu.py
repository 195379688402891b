"""GPU: fused RVQ dequant-GEMV (batch 1) against the oracle's reconstruction.

Two references:
* fp64 product of the oracle-reconstructed fp32 weights: the table-based
  GEMV computes that sum exactly up to fp32 rounding -> rel. error <= 2e-5;
* the reference's path, F.linear on the weight rounded to bf16 (what the
  slot holds): differs by the bf16 rounding of W -> rel. error <= 1e-2
  (the tolerance the linear microbenchmark is specified with).
"""

import numpy as np
import pytest
import torch

from oracle.rvq_oracle import OUT_F32, RVQEntryNP, decode_rvq
from rvq_b200 import synthetic
from rvq_b200.gemv import GemvPlan, gemv_supported, interleave_codes, rvq_linear

pytestmark = pytest.mark.gpu


def oracle_w(entry, cb):
    numel = int(np.prod(entry["shape"]))
    e = RVQEntryNP(indices=entry["indices"].numpy(), codebook=cb.float().numpy(),
                   scales=entry["scales"].float().numpy(), tail=entry["tail"].float().numpy(), d=8,
                   group_size=int(entry["group_size"]), trimmed_numel=int(entry["trimmed_numel"]),
                   numel=numel)
    return decode_rvq(e, OUT_F32).reshape(entry["shape"]).astype(np.float64)


def to_dev(entry, device):
    return {k: (v.to(device) if torch.is_tensor(v) else v) for k, v in entry.items()}


def rel_err(got, want):
    got = np.asarray(got, np.float64)
    return float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30))


@pytest.mark.parametrize("rows,cols,group", [
    (9728, 2560, None),          # config-1 gate projection, per-row scales
    (2560, 9728, None),          # down projection (38 column tiles)
    (1024, 2560, 128),           # compressor default: group 128 -> 16 vectors per scale
    (333, 520, None),            # ragged last column tile (65 groups), odd row count
    (64, 64, 64),
])
@pytest.mark.parametrize("x_dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("layout", ["planes", "interleaved"])
def test_gemv_matches_reconstruction(rows, cols, group, x_dtype, layout, cuda_device):
    g = torch.Generator().manual_seed(rows * 7 + cols)
    cb = synthetic.make_codebook(4, 256, 8, g)
    entry = synthetic.make_rvq_entry(rows, cols, g, group_size=group)
    assert gemv_supported(entry)
    x = torch.randn(cols, generator=g).to(x_dtype)
    dev_entry = to_dev(entry, cuda_device)
    if layout == "interleaved":
        dev_entry["codes_il"] = interleave_codes(dev_entry["indices"])
    y = rvq_linear(x.to(cuda_device), dev_entry, cb.to(cuda_device, torch.float32), out_dtype=torch.float32)
    torch.cuda.synchronize()
    w = oracle_w(entry, cb)
    xd = x.float().numpy().astype(np.float64)
    exact = w @ xd
    assert rel_err(y.cpu().numpy(), exact) <= 2e-5
    # the reference path: bf16 slot weight, then the matmul
    w_bf16 = torch.from_numpy(w.astype(np.float32)).to(torch.bfloat16).double().numpy()
    assert rel_err(y.cpu().numpy(), w_bf16 @ xd) <= 1e-2


def test_gemv_is_deterministic_and_reusable(cuda_device):
    g = torch.Generator().manual_seed(3)
    cb = synthetic.make_codebook(4, 256, 8, g).to(cuda_device)
    entry = to_dev(synthetic.make_rvq_entry(4096, 2560, g), cuda_device)
    x = torch.randn(2560, generator=g).to(cuda_device, torch.bfloat16)
    y = torch.empty(4096, dtype=torch.float32, device=cuda_device)
    plan = GemvPlan([(entry, cb, x, y)])
    outs = []
    for _ in range(3):
        plan.launch()
        outs.append(y.clone())
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])


def test_interleave_codes_layout(cuda_device):
    g = torch.Generator().manual_seed(8)
    idx = torch.randint(0, 256, (4, 1000), dtype=torch.uint8, generator=g)
    il = interleave_codes(idx.to(cuda_device)).cpu().view(1000, 4)
    assert torch.equal(il, idx.t().contiguous())


def test_gemv_multi_job_shared_x(cuda_device):
    """q, k, v of one 2560-wide layer in one launch, sharing x."""
    g = torch.Generator().manual_seed(4)
    cbs = synthetic.make_family_codebooks(g)
    ents = {name: synthetic.make_rvq_entry(rows, 2560, g, codebook_id=fam)
            for name, rows, fam in (("q", 4096, "attn_q_proj"), ("k", 1024, "attn_k_proj"),
                                    ("v", 1024, "attn_v_proj"))}
    x = torch.randn(2560, generator=g).to(torch.bfloat16)
    xd = x.to(cuda_device)
    ys = {n: torch.empty(int(e["shape"][0]), dtype=torch.bfloat16, device=cuda_device) for n, e in ents.items()}
    plan = GemvPlan([(to_dev(e, cuda_device), cbs[e["codebook_id"]].to(cuda_device), xd, ys[n])
                     for n, e in ents.items()])
    plan.launch()
    torch.cuda.synchronize()
    for n, e in ents.items():
        want = oracle_w(e, cbs[e["codebook_id"]]) @ x.float().numpy().astype(np.float64)
        assert rel_err(ys[n].float().cpu().numpy(), want) <= 5e-3, n   # bf16 output rounding


def test_gemv_rejects_unsupported(cuda_device):
    g = torch.Generator().manual_seed(5)
    entry = synthetic.make_rvq_entry(64, 64, g, stages=3)
    assert not gemv_supported(entry)
    with pytest.raises(NotImplementedError):
        GemvPlan([(to_dev(entry, cuda_device), synthetic.make_codebook(3, 256, 8, g).to(cuda_device),
                   torch.zeros(64, device=cuda_device), torch.zeros(64, device=cuda_device))])
