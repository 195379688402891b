"""GPU: the tcgen05 prefill GEMM (weight decoded into shared memory) against
decode-into-slot + cuBLAS on the same bit-exact bf16 weight.

Both multiply the same bf16 values with fp32 accumulation and round to bf16;
only the accumulation order differs, so results agree to ~1e-3 relative.
"""

import pytest
import torch

from rvq_b200 import synthetic
from rvq_b200.engine import decode_to_tensor
from rvq_b200.gemm import GemmPlan, rvq_matmul, take_timeout
from rvq_b200.gemv import interleave_codes

pytestmark = pytest.mark.gpu


def dev_entry(entry, device):
    e = {k: (v.to(device) if torch.is_tensor(v) else v) for k, v in entry.items()}
    e["codes_il"] = interleave_codes(e["indices"])
    return e


@pytest.mark.parametrize("m,n,k,group", [(128, 256, 64, None), (256, 512, 2560, None), (200, 1024, 256, 128),
                                         (2048, 9728, 2560, None), (77, 2560, 9728, None)])
def test_prefill_gemm_matches_decode_then_matmul(m, n, k, group, cuda_device):
    g = torch.Generator().manual_seed(m + n + k)
    cb = synthetic.make_codebook(4, 256, 8, g)
    entry = dev_entry(synthetic.make_rvq_entry(n, k, g, group_size=group), cuda_device)
    cbd = {"global_2d": cb.to(cuda_device, torch.float32)}
    w = decode_to_tensor(entry, cbd, cuda_device, torch.bfloat16)           # bit-exact slot weight
    x = torch.randn(m, k, generator=g).to(cuda_device, torch.bfloat16)
    y = rvq_matmul(x, entry, cbd["global_2d"])
    torch.cuda.synchronize()
    assert not take_timeout()
    ref32 = x.float() @ w.float().t()
    ref = torch.matmul(x, w.t())
    rel32 = float((y.float() - ref32).norm() / ref32.norm())
    rel = float((y.float() - ref.float()).norm() / ref.float().norm())
    assert rel32 < 5e-3, rel32
    assert rel < 5e-3, rel
    # most outputs equal cuBLAS's bf16 result, the rest differ by ~1 ulp
    assert float((y.float() - ref.float()).abs().max() / ref.float().abs().max()) < 2e-2


def test_prefill_gemm_is_deterministic(cuda_device):
    g = torch.Generator().manual_seed(5)
    cb = synthetic.make_codebook(4, 256, 8, g).to(cuda_device, torch.float32)
    entry = dev_entry(synthetic.make_rvq_entry(1024, 2560, g), cuda_device)
    x = torch.randn(384, 2560, generator=g).to(cuda_device, torch.bfloat16)
    y = torch.empty(384, 1024, dtype=torch.bfloat16, device=cuda_device)
    plan = GemmPlan(entry, cb, x, y)
    plan.launch()
    y0 = y.clone()
    for _ in range(3):
        plan.launch()
    torch.cuda.synchronize()
    assert torch.equal(y, y0)
