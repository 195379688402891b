"""GPU: the slot kernel (quad-layout codes, rvq_slot_kernel) against the
planar path and the oracle.

A layer plan repacks every eligible entry (4 stages of 256 uint8 codes, an
fp16-exact codebook, a bf16 slot, fp16 scales, 4 | vectors per scale) into the
quad layout once; the slot kernel must then write exactly the bits the
planar path and the oracle produce -- including an entry whose last
128-vector tile is partial -- and nothing outside each slot tensor.
Ineligible entries in the same layer keep the planar path."""

import numpy as np
import pytest
import torch

from oracle.rvq_oracle import OUT_BF16, RVQEntryNP, decode_rvq_bits
from rvq_b200 import synthetic
from rvq_b200.engine import LayerDecodePlan

pytestmark = pytest.mark.gpu

SHAPES = [
    ("a", 4096, 2560, None),     # per-row scales (320 vectors each), whole 128-vector tiles
    ("b", 100, 96, 32),          # 4 vectors per scale, 1200 vectors: a partial last tile
    ("c", 1000, 64, 64),         # 8 vectors per scale, 8000 vectors: a partial last tile
    ("d", 333, 520, None),       # 65 vectors per scale: not a multiple of 4 -> planar path
]


def _layer(device, exact_cb=True, seed=5):
    g = torch.Generator().manual_seed(seed)
    cb = synthetic.make_codebook(4, 256, 8, g).float()
    if not exact_cb:
        cb = cb * (1 + 1e-6 * torch.randn(cb.shape, generator=g))
    items, host = [], {}
    for name, r, c, group in SHAPES:
        e = synthetic.make_rvq_entry(r, c, g, group_size=group, codebook_id="cb")
        host[name] = e
        items.append((name, {k: (v.to(device) if torch.is_tensor(v) else v) for k, v in e.items()}))
    return items, host, {"cb": cb.to(device)}, cb


def _decode(items, cbs, device, quad):
    bufs, outs = {}, {}
    for name, e in items:
        n = int(np.prod(e["shape"]))
        buf = torch.full((n + 64,), 3.0, dtype=torch.bfloat16, device=device)
        bufs[name] = buf
        outs[name] = buf[:n].view(tuple(e["shape"]))
    LayerDecodePlan(items, cbs, outs, quad_codes=quad).launch()
    torch.cuda.synchronize()
    return bufs


@pytest.mark.parametrize("exact_cb", [True, False])
def test_slot_kernel_matches_planes_and_oracle(exact_cb, cuda_device):
    items, host, cbs, cb = _layer(cuda_device, exact_cb)
    quad = _decode(items, cbs, cuda_device, True)
    planar = _decode(items, cbs, cuda_device, False)
    for name, e in host.items():
        n = int(np.prod(e["shape"]))
        assert torch.equal(quad[name], planar[name]), name
        assert torch.all(quad[name][n:] == 3.0), name
        ent = RVQEntryNP(indices=e["indices"].numpy(), codebook=cb.numpy(), scales=e["scales"].float().numpy(),
                         tail=e["tail"].float().numpy(), d=8, group_size=int(e["group_size"]),
                         trimmed_numel=int(e["trimmed_numel"]), numel=n)
        got = quad[name][:n].cpu().view(torch.int16).numpy().view(np.uint16)
        assert np.array_equal(got, decode_rvq_bits(ent, OUT_BF16)), name


def test_quad_layout(cuda_device):
    """rvq_quad_codes against a host restatement: byte 4 k + j of quad q is
    the stage-k code of vector 4 q + j; zeros up to a whole 128-vector tile."""
    import ctypes
    from rvq_b200 import _native
    lib = _native.load()
    lib.rvq_quad_codes_bytes.restype = ctypes.c_int64
    lib.rvq_quad_codes_bytes.argtypes = [ctypes.c_int64]
    lib.rvq_quad_codes.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]
    for nvec in (1, 131, 1200, 4096):
        planes = torch.randint(0, 256, (4, nvec), dtype=torch.uint8, generator=torch.Generator().manual_seed(nvec))
        nb = int(lib.rvq_quad_codes_bytes(nvec))
        assert nb == -(-nvec // 128) * 512
        out = torch.full((nb,), 7, dtype=torch.uint8, device=cuda_device)
        dp = planes.to(cuda_device)
        assert lib.rvq_quad_codes(dp.data_ptr(), nvec, nvec, out.data_ptr(), None) == 0
        torch.cuda.synchronize()
        want = np.zeros((nb // 16, 4, 4), np.uint8)
        p = planes.numpy()
        for n in range(nvec):
            want[n // 4, :, n % 4] = p[:, n]
        assert np.array_equal(out.cpu().numpy().reshape(-1, 4, 4), want)
