"""C-ABI library: loads, exports what include/rvq_b200.h declares, and its
host-side logic behaves (no GPU needed, no kernel launched)."""

import ctypes
import os
import re

import numpy as np
import pytest

from rvq_b200 import _native

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER_DIR = os.path.join(REPO, "include")


def declared_functions():
    names = set()
    for fn in os.listdir(HEADER_DIR):
        if not fn.endswith(".h"):
            continue
        text = open(os.path.join(HEADER_DIR, fn)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"^\s*[A-Za-z_][\w\s\*]*?\b(rvq_\w+)\s*\(", text, flags=re.M):
            names.add(m.group(1))
    return sorted(names)


@pytest.fixture(scope="module")
def lib():
    return _native.load()


def test_header_declares_entry_points():
    names = declared_functions()
    for required in ("rvq_decode", "rvq_decode_layer", "rvq_available", "rvq_check_entry"):
        assert required in names, names


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"


def test_struct_layout_matches_header(lib):
    # 5 pointers + 5 int64 + 8 int32
    assert ctypes.sizeof(_native.RvqEntry) == 5 * 8 + 5 * 8 + 8 * 4
    assert ctypes.sizeof(_native.RvqCopy) == 24


def test_step_struct_layouts():
    from rvq_b200 import step
    assert ctypes.sizeof(step.RvqVec) == 24
    assert ctypes.sizeof(step.RvqNormArgs) == 8 + 24 + 4 * 8 + 8 + 4 + 4 + 8 + 8 + 4 + 4
    assert ctypes.sizeof(step.RvqAttnArgs) == 3 * 24 + 8 * 8 + 4 * 4 + 4 * 4
    from rvq_b200 import gemv
    assert ctypes.sizeof(gemv.RvqGemvTileJob) == ctypes.sizeof(_native.RvqEntry) + 2 * 24 + 3 * 8
    from rvq_b200 import gemm
    # entry + x, y + rows, cols, tokens + x_kind, y_kind, exact, reserved
    assert ctypes.sizeof(gemm.RvqGemvBatchJob) == ctypes.sizeof(_native.RvqEntry) + 2 * 8 + 3 * 8 + 4 * 4
    assert gemv.tiles_count(2560) == 10 and gemv.tiles_count(9728) == 38 and gemv.tiles_count(520) == 3
    lib = gemv._tiles_lib()
    assert lib.rvq_tile_codes_bytes(9728, 2560) == 10 * 9728 * 128
    assert lib.rvq_tile_codes_bytes(5, 520) == 3 * 5 * 128
    assert lib.rvq_tile_codes_bytes(5, 12) == 0


def test_step_calls_reject_bad_arguments(lib):
    """Host-side checks run before any launch (no device needed)."""
    from rvq_b200 import step
    step._lib()
    assert lib.rvq_step_norm(None, None) == _native.RVQ_ERR_INVALID
    a = step.RvqNormArgs(8, step.RvqVec(None, 0, 0, 0), None, None, 8, 8, 1 << 20, 1e-6, 0)
    assert lib.rvq_step_norm(ctypes.byref(a), None) == _native.RVQ_ERR_UNSUPPORTED
    a.hidden = 64
    a.add = step.RvqVec(8, 32, 1, _native.RVQ_BF16)            # wrong length
    assert lib.rvq_step_norm(ctypes.byref(a), None) == _native.RVQ_ERR_INVALID
    v = step.RvqVec(8, 128, 1, _native.RVQ_BF16)
    at = step.RvqAttnArgs(v, v, v, 8, 8, 8, 8, 8, 8, 8, 8, 3, 2, 64, 16, 1e-6, 0.1, 1.0, 0)
    assert lib.rvq_step_attention(ctypes.byref(at), None) == _native.RVQ_ERR_INVALID   # 3 % 2 != 0
    at.n_heads, at.n_kv, at.head_dim = 2, 2, 96
    at.q = at.k = at.v = step.RvqVec(8, 192, 1, _native.RVQ_BF16)
    assert lib.rvq_step_attention(ctypes.byref(at), None) == _native.RVQ_ERR_UNSUPPORTED
    at.n_heads, at.n_kv, at.head_dim = 64, 2, 64                                   # 32 heads per kv head
    assert lib.rvq_step_attention(ctypes.byref(at), None) == _native.RVQ_ERR_UNSUPPORTED
    g = step.RvqVec(8, 100, 1, _native.RVQ_BF16)
    u = step.RvqVec(8, 99, 1, _native.RVQ_BF16)
    assert lib.rvq_step_silu_mul(ctypes.byref(g), ctypes.byref(u), 8, None) == _native.RVQ_ERR_INVALID


def test_tp_push_struct_and_host_checks(lib):
    """Peer-exchange entry points: struct layout, CTA count, argument checks."""
    from rvq_b200 import step, tp
    tp._lib()
    assert ctypes.sizeof(tp.RvqTpPushArgs) == 24 + 2 * 8 * tp.RVQ_MAX_TP + 8 + 4 + 4
    assert tp.push_ctas(5120) == 40 and tp.push_ctas(128) == 1 and tp.push_ctas(129) == 2
    a = tp.RvqTpPushArgs()
    a.src = step.RvqVec(8, 64, 1, _native.RVQ_BF16)
    a.n, a.rank, a.tp = 64, 0, 2
    a.dst[0], a.arrivals[0] = 8, 8                                  # rank 1's pointers missing
    assert lib.rvq_tp_push(ctypes.byref(a), None) == _native.RVQ_ERR_INVALID
    a.tp = tp.RVQ_MAX_TP + 1
    assert lib.rvq_tp_push(ctypes.byref(a), None) == _native.RVQ_ERR_INVALID
    a.tp, a.rank = 2, 2
    assert lib.rvq_tp_push(ctypes.byref(a), None) == _native.RVQ_ERR_INVALID
    n = step.RvqNormArgs(8, step.RvqVec(8, 64, 2, _native.RVQ_F32), None, None, 8, 8, 64, 1e-6, 0)
    n.arrivals = 8                                                   # no consumed counter
    assert lib.rvq_step_norm(ctypes.byref(n), None) == _native.RVQ_ERR_INVALID


def test_status_strings(lib):
    assert _native.status_string(0) == "ok"
    for s in range(1, 6):
        assert _native.status_string(s) != "unknown status"


def test_fastdiv_host_mirror(lib):
    rng = np.random.default_rng(0)
    divisors = [1, 2, 3, 5, 7, 16, 20, 40, 320, 512, 640, 1216, 3200, 65535, 65536, 1 << 20,
                (1 << 31) - 1, (1 << 31) + 12345, (1 << 32) - 1]
    divisors += list(rng.integers(1, 1 << 32, size=40, dtype=np.uint64))
    for d in divisors:
        d = int(d)
        ns = [0, 1, d - 1, d, d + 1, 2 * d - 1, (1 << 32) - 1, (1 << 31), (1 << 31) - 1]
        ns += list(rng.integers(0, 1 << 32, size=200, dtype=np.uint64))
        for n in ns:
            n = int(n) & 0xFFFFFFFF
            assert lib.rvq_test_fastdiv(d, n) == n // d, (d, n)


def _fake_entry(**kw):
    e = _native.RvqEntry()
    e.indices, e.codebook, e.scales, e.tail, e.out = 0x1000, 0x2000, 0x3000, 0, 0x4000
    e.nvec, e.stage_stride, e.group_vecs, e.trimmed, e.tail_numel = 1024, 1024, 16, 8192, 0
    e.stages, e.ncodes, e.d = 4, 256, 8
    e.index_kind, e.codebook_kind, e.scale_kind = _native.RVQ_U8, _native.RVQ_F32, _native.RVQ_F16
    e.tail_kind, e.out_kind = _native.RVQ_BF16, _native.RVQ_BF16
    for k, v in kw.items():
        setattr(e, k, v)
    return e


@pytest.mark.parametrize("field,value,status", [
    ("d", 4, _native.RVQ_ERR_UNSUPPORTED),
    ("out_kind", _native.RVQ_U8, _native.RVQ_ERR_UNSUPPORTED),
    ("index_kind", _native.RVQ_F16, _native.RVQ_ERR_UNSUPPORTED),
    ("stages", 0, _native.RVQ_ERR_INVALID),
    ("ncodes", 300, _native.RVQ_ERR_INVALID),          # > 256 with uint8 indices
    ("group_vecs", 0, _native.RVQ_ERR_INVALID),
    ("trimmed", 1024 * 8 + 1, _native.RVQ_ERR_INVALID),
    ("stage_stride", 1000, _native.RVQ_ERR_INVALID),
    ("out", 0, _native.RVQ_ERR_INVALID),
    ("tail_numel", 5, _native.RVQ_ERR_INVALID),          # tail pointer is NULL
    ("codebook", 0x2004, _native.RVQ_ERR_INVALID),       # not 16-byte aligned
    ("nvec", 1 << 31, _native.RVQ_ERR_TOO_LARGE),
])
def test_check_entry_rejects(lib, field, value, status):
    e = _fake_entry(**{field: value})
    if field == "nvec":
        e.stage_stride = value
    assert lib.rvq_check_entry(ctypes.byref(e)) == status


def test_check_entry_accepts_valid(lib):
    assert lib.rvq_check_entry(ctypes.byref(_fake_entry())) == 0
    e = _fake_entry(index_kind=_native.RVQ_I16, ncodes=512)
    assert lib.rvq_check_entry(ctypes.byref(e)) == 0


def test_layer_call_rejects_too_many_jobs(lib):
    arr = (_native.RvqEntry * 40)(*[_fake_entry() for _ in range(40)])
    assert lib.rvq_decode_layer(arr, 40, None, 0, None) == _native.RVQ_ERR_INVALID


def test_no_device_means_unavailable():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    from rvq_b200 import triton_decode_kernels as tdk
    assert tdk.triton_available() is False
    assert _native.load().rvq_available() == 0
    with pytest.raises(RuntimeError):
        import torch as _t
        entry = {"d": 8, "group_size": 8, "trimmed_numel": 8, "method": "rvq_groupwise"}
        tdk.decode_rvq_triton_into(entry, _t.zeros(1, 256, 8), _t.zeros(8))


def test_int8_entry_checks(lib):
    """Host-side validation of rvq_int8_entry (no device memory touched)."""
    assert ctypes.sizeof(_native.RvqInt8Entry) == 4 * 8 + 3 * 8 + 4 * 4
    e = _native.RvqInt8Entry()
    e.q, e.scales, e.out = 0x1000, 0x2000, 0x3000
    e.trimmed, e.group_size, e.tail_numel = 4096, 128, 0
    e.scale_kind, e.tail_kind, e.out_kind = _native.RVQ_F16, _native.RVQ_BF16, _native.RVQ_BF16
    assert lib.rvq_check_int8_entry(ctypes.byref(e)) == _native.RVQ_OK
    e.trimmed = 4000                                   # not a multiple of the group size
    assert lib.rvq_check_int8_entry(ctypes.byref(e)) == _native.RVQ_ERR_INVALID
    e.trimmed, e.out_kind = 4096, _native.RVQ_U8
    assert lib.rvq_check_int8_entry(ctypes.byref(e)) == _native.RVQ_ERR_UNSUPPORTED
    e.out_kind, e.tail_numel, e.tail = _native.RVQ_BF16, 5, None
    assert lib.rvq_check_int8_entry(ctypes.byref(e)) == _native.RVQ_ERR_INVALID
    e.tail_numel, e.trimmed = 0, 1 << 31
    assert lib.rvq_check_int8_entry(ctypes.byref(e)) == _native.RVQ_ERR_TOO_LARGE
    assert lib.rvq_decode_layer_mixed(None, 0, None, 40, None, 0, None) == _native.RVQ_ERR_INVALID


def test_persist_structs_and_host_checks(lib):
    """The persistent decode step's structs and its argument checks (no device
    memory touched; without a GPU the planner reports nothing plannable)."""
    import torch
    from rvq_b200 import persist
    assert ctypes.sizeof(persist.RvqPersistLayer) == 7 * ctypes.sizeof(_native.RvqEntry) + 6 * 8
    # 12 four-byte fields, 17 pointers
    assert ctypes.sizeof(persist.RvqPersistModel) == 12 * 4 + 17 * 8
    assert persist.SYNC_WORDS == 1024
    plib = persist._lib()
    assert plib.rvq_persist_step(None, None) == _native.RVQ_ERR_INVALID
    assert plib.rvq_persist_step(ctypes.c_void_p(0x1008), None) == _native.RVQ_ERR_INVALID   # not 16-byte aligned
    assert plib.rvq_persist_plan(None, None, None, 0) == _native.RVQ_ERR_INVALID
    if not torch.cuda.is_available():
        m = persist.RvqPersistModel()
        layers = (persist.RvqPersistLayer * 1)()
        assert plib.rvq_persist_plan_bytes(ctypes.byref(m), layers) == 0
        buf = (ctypes.c_char * 16)()
        assert plib.rvq_persist_plan(ctypes.byref(m), layers, buf, 16) == _native.RVQ_ERR_UNAVAILABLE
        assert plib.rvq_persist_step(ctypes.c_void_p(0x1000), None) == _native.RVQ_ERR_UNAVAILABLE
