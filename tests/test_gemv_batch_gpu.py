"""GPU: rvq_gemv_batch (fused GEMM on tcgen05, batches and prompts) against the oracle.

In exact mode the kernel multiplies x by the bit-exact bf16 slot weights
(the oracle's reconstruction rounded to nearest even) with fp32 accumulation
in TMEM, then rounds y to bf16.  So y agrees with the fp64 product of x and
the oracle's bf16 weights to the bf16 output rounding (2^-9 relative per
element; the norm-wise bound used here is 4e-3).  The fast mode sums the
stage codewords in fp16 before scaling and rounding to bf16, so a weight may
differ from the slot's by one bf16 ulp; the same bound holds.  Both are well
inside config 3's 1e-2 tolerance against the reference's
reconstruct-then-matmul, which is also checked.
"""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle.rvq_oracle import OUT_BF16, RVQEntryNP, bf16_bits_to_f32, decode_rvq_bits
from rvq_b200 import synthetic
from rvq_b200.gemm import BatchGemvPlan, take_batch_timeout
from rvq_b200.gemv import tile_codes

pytestmark = pytest.mark.gpu

TOL = 4e-3


def oracle_w_bf16(entry, cb):
    numel = int(np.prod(entry["shape"]))
    e = RVQEntryNP(indices=entry["indices"].numpy(), codebook=cb.float().numpy(),
                   scales=entry["scales"].float().numpy(), tail=entry["tail"].float().numpy(), d=8,
                   group_size=int(entry["group_size"]), trimmed_numel=int(entry["trimmed_numel"]), numel=numel)
    return bf16_bits_to_f32(decode_rvq_bits(e, OUT_BF16)).reshape(entry["shape"]).astype(np.float64)


def rel(got, want):
    return float(np.linalg.norm(np.asarray(got, np.float64) - want) / max(np.linalg.norm(want), 1e-30))


@pytest.mark.parametrize("rows,cols,tokens,group,cb_dtype", [
    (9728, 2560, 1, None, torch.float32),      # config-3 gate, batch 1
    (9728, 2560, 8, None, torch.float32),      # batch 8
    (9728, 2560, 64, None, torch.float16),     # batch 64, fp16 codebook
    (2560, 9728, 8, None, torch.float32),      # down projection: 152 chunks per row tile
    (1024, 2560, 16, None, torch.float32),     # 8 row tiles cut into ~19 pieces each
    (333, 520, 5, None, torch.float32),        # ragged rows and a partial last chunk
    (8, 8, 1, 8, torch.float32),               # one vector
    (3000, 1000, 17, 40, torch.float32),       # 5 vectors per scale
    (200, 512, 256, None, torch.float32),      # 256 tokens: two blocks of 128
    (1000, 1024, 300, None, torch.float32),    # 300 tokens: two blocks of 160 (the last partial)
    (9728, 2560, 128, None, torch.float16),    # 128 tokens: one block
    (2560, 2560, 150, None, torch.float16),    # 150 tokens: one block of 160
    (2560, 9728, 64, 128, torch.float16),      # down projection, 64 tokens, group-128 scales
    (640, 512, 192, None, torch.float32),      # 192 tokens: one block, 512 TMEM columns
    (9728, 2560, 2048, None, torch.float16),   # a 2048-token prompt on the gate projection
    (2048, 2560, 8, None, "f32_not_f16"),      # codebook fp16 cannot hold: global fp32 reads
    (2048, 2560, 8, 128, torch.float16),       # group 128 (the compressor default): 2 chunks per scale
])
@pytest.mark.parametrize("exact", [False, True], ids=["fast", "exact"])
def test_batch_matches_bf16_reconstruction(rows, cols, tokens, group, cb_dtype, exact, cuda_device):
    g = torch.Generator().manual_seed(rows * 7 + cols + tokens)
    cb = synthetic.make_codebook(4, 256, 8, g)
    if cb_dtype == "f32_not_f16":
        cb = cb.float() * (1 + 1e-6 * torch.randn(cb.shape, generator=g))
        cb_dtype = torch.float32
    entry = synthetic.make_rvq_entry(rows, cols, g, group_size=group)
    x = torch.randn(tokens, cols, generator=g).to(torch.bfloat16)
    dev = {k: (v.to(cuda_device) if torch.is_tensor(v) else v) for k, v in entry.items()}
    dev["codes_tiled"] = tile_codes(dev["indices"], rows, cols)
    y = torch.full((tokens, rows), float("nan"), dtype=torch.bfloat16, device=cuda_device)
    plan = BatchGemvPlan(dev, cb.to(cuda_device, cb_dtype), x.to(cuda_device), y, exact=exact)
    plan.launch()
    torch.cuda.synchronize()
    w = oracle_w_bf16(entry, cb)
    got = y.float().cpu().numpy()
    assert not np.isnan(got).any()
    wd = torch.from_numpy(w).to(cuda_device)
    if tokens <= 256:
        want = x.double().numpy() @ w.T
    else:                                       # large: the fp64 product on the GPU
        want = (x.to(cuda_device).double() @ wd.t()).cpu().numpy()
    assert rel(got, want) <= TOL
    # the reference's reconstruct + F.linear on the same weights (config 3: 1e-2)
    lin = F.linear(x.to(cuda_device), wd.to(torch.bfloat16)).float().cpu().numpy()
    assert rel(got, lin) <= 1e-2
    # deterministic across launches (tickets reset, pieces added in a fixed order)
    first = y.clone()
    for _ in range(3):
        plan.launch()
    torch.cuda.synchronize()
    assert torch.equal(y, first)
    assert not take_batch_timeout()
