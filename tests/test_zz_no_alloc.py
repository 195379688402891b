"""GPU: rvq_gemv_noalloc, the GEMV entry point that allocates nothing.

It exists for callers that cannot allocate device memory (a serving process
whose memory budget is fixed at start-up, a plug-in inside a runtime that owns
every device allocation): its workspace is a fixed array in the library's
device memory.  This file runs last so that, if it fails, a run that stops at
the first failure has already run every other test; it must also pass when
run alone in a fresh process.
"""

import ctypes

import numpy as np
import pytest
import torch

from rvq_b200 import _native, synthetic
from rvq_b200.gemv import GemvPlan, RvqGemvJob, _lib, interleave_codes

pytestmark = pytest.mark.gpu


def bind(lib):
    lib.rvq_gemv_noalloc.restype = ctypes.c_int
    lib.rvq_gemv_noalloc.argtypes = [ctypes.POINTER(RvqGemvJob), ctypes.c_int, ctypes.c_void_p]
    lib.rvq_gemv_noalloc_max_workspace.restype = ctypes.c_size_t
    lib.rvq_gemv_noalloc_max_workspace.argtypes = []
    return lib


def rel_err(a, b):
    a = a.double().cpu().numpy()
    b = b.double().cpu().numpy()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def to_dev(entry, device):
    return {k: (v.to(device) if torch.is_tensor(v) else v) for k, v in entry.items()}


@pytest.mark.parametrize("shape,interleaved", [((9728, 2560), True), ((2560, 9728), False),
                                               ((333, 520), False)])
def test_noalloc_matches_allocating_entry_point(shape, interleaved, cuda_device):
    lib = bind(_lib())
    g = torch.Generator().manual_seed(shape[0])
    cb = synthetic.make_codebook(4, 256, 8, g).to(cuda_device, torch.float32)
    entry = to_dev(synthetic.make_rvq_entry(shape[0], shape[1], g), cuda_device)
    if interleaved:
        entry["codes_il"] = interleave_codes(entry["indices"])
    x = torch.randn(shape[1], generator=g).to(cuda_device, torch.bfloat16)
    y_ref = torch.empty(shape[0], dtype=torch.float32, device=cuda_device)
    GemvPlan([(entry, cb, x, y_ref)]).launch()           # existing entry point, own workspace

    for call in range(2):                                 # two calls in a row share the array
        y = torch.full((shape[0],), float("nan"), dtype=torch.float32, device=cuda_device)
        plan = GemvPlan([(entry, cb, x, y)])              # only to build the C job descriptors
        stream = torch.cuda.current_stream(cuda_device).cuda_stream
        rc = lib.rvq_gemv_noalloc(plan.jobs, plan.n, ctypes.c_void_p(stream))
        assert rc == _native.RVQ_OK, _native.status_string(rc)
        torch.cuda.synchronize()
        assert not torch.isnan(y).any(), call
        assert rel_err(y, y_ref) <= 2e-5, call           # the GEMV tests' tolerance
        assert torch.equal(y, y_ref), call                # same kernels, same plan: identical


def test_noalloc_rejects_jobs_beyond_its_workspace(cuda_device):
    """A GEMV whose workspace exceeds the fixed array is refused before any
    launch (the 25600-wide down projection needs 100 tables of 128 KB)."""
    lib = bind(_lib())
    limit = int(lib.rvq_gemv_noalloc_max_workspace())
    assert limit == 8 << 20
    g = torch.Generator().manual_seed(1)
    entry = synthetic.make_rvq_entry(64, 25600, g)
    cb = synthetic.make_codebook(4, 256, 8, g).to(cuda_device)
    x = torch.zeros(25600, dtype=torch.bfloat16, device=cuda_device)
    y = torch.zeros(64, dtype=torch.float32, device=cuda_device)
    plan = GemvPlan([(to_dev(entry, cuda_device), cb, x, y)])
    assert plan.workspace_bytes > limit
    rc = lib.rvq_gemv_noalloc(plan.jobs, plan.n, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == _native.RVQ_ERR_TOO_LARGE


def test_noalloc_calls_allocate_nothing(cuda_device):
    """After the first call on the device (which looks up the array's
    address), further calls change neither torch's allocator statistics nor
    the device's free memory."""
    lib = bind(_lib())
    g = torch.Generator().manual_seed(7)
    cb = synthetic.make_codebook(4, 256, 8, g).to(cuda_device, torch.float32)
    entry = to_dev(synthetic.make_rvq_entry(4096, 2560, g), cuda_device)
    x = torch.randn(2560, generator=g).to(cuda_device, torch.bfloat16)
    y = torch.zeros(4096, dtype=torch.float32, device=cuda_device)
    plan = GemvPlan([(entry, cb, x, y)])
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    assert lib.rvq_gemv_noalloc(plan.jobs, plan.n, stream) == _native.RVQ_OK       # warm-up call
    torch.cuda.synchronize()
    allocated, reserved = torch.cuda.memory_allocated(cuda_device), torch.cuda.memory_reserved(cuda_device)
    free_before = torch.cuda.mem_get_info(cuda_device)[0]
    for _ in range(5):
        assert lib.rvq_gemv_noalloc(plan.jobs, plan.n, stream) == _native.RVQ_OK
    torch.cuda.synchronize()
    assert torch.cuda.memory_allocated(cuda_device) == allocated
    assert torch.cuda.memory_reserved(cuda_device) == reserved
    assert torch.cuda.mem_get_info(cuda_device)[0] == free_before
