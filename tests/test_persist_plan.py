"""The persistent decode step's host-side plan, checked without a GPU
(rvq_persist_plan_for: the plan for a given CTA count, nothing launched).

The plan holds, per layer and GEMV phase, the unit split of the table GEMV
(rvq_gemv_tiles' planner) over the CTAs.  Here: every (job, tile, row) of
every phase is covered by exactly one unit, each CTA's unit range lies
inside its phase, and every offset of the plan stays inside it.
"""

import ctypes
import struct

import numpy as np
import pytest

from rvq_b200 import _native, persist

HEAD_BYTES = 184 + 4 * 4 + 5 * 8           # the model, 4 int32, 5 int64 offsets


def fake_entry(rows, cols, base):
    e = _native.RvqEntry()
    nvec = rows * cols // 8
    e.indices, e.codebook, e.scales, e.tail, e.out = base, base + 0x100000, base + 0x200000, 0, base + 0x300000
    e.nvec, e.stage_stride, e.group_vecs, e.trimmed, e.tail_numel = nvec, nvec, cols // 8, nvec * 8, 0
    e.stages, e.ncodes, e.d = 4, 256, 8
    e.index_kind, e.codebook_kind, e.scale_kind = _native.RVQ_U8, _native.RVQ_F16, _native.RVQ_F16
    e.tail_kind, e.out_kind = _native.RVQ_BF16, _native.RVQ_BF16
    return e


def fake_model(n_layers, hidden, inter, n_heads, n_kv, max_len=256):
    m = persist.RvqPersistModel()
    m.n_layers, m.hidden, m.intermediate, m.n_heads, m.n_kv, m.head_dim = n_layers, hidden, inter, n_heads, n_kv, 128
    m.max_len, m.vocab, m.eps, m.scaling, m.valid_bias = max_len, 1000, 1e-6, 128 ** -0.5, 1.0
    ptr = 0x7000_0000
    for name, _ in persist.RvqPersistModel._fields_[12:]:
        setattr(m, name, ptr)
        ptr += 0x10000
    qd, kd = n_heads * 128, n_kv * 128
    shapes = [(qd, hidden), (kd, hidden), (kd, hidden), (hidden, qd), (inter, hidden), (inter, hidden),
              (hidden, inter)]
    layers = (persist.RvqPersistLayer * n_layers)()
    for l in range(n_layers):
        for p, (r, c) in enumerate(shapes):
            layers[l].proj[p] = fake_entry(r, c, 0x1_0000_0000 * (l + 1) + 0x1000_0000 * p)
        for k, name in enumerate(("input_norm", "post_norm", "q_norm", "k_norm", "k_cache", "v_cache")):
            setattr(layers[l], name, 0x9000_0000 + 0x1000 * (6 * l + k))
    return m, layers, shapes


PHASE_JOBS = [(0, 1, 2), (3,), (4, 5), (6,)]       # projections of each GEMV phase


@pytest.mark.parametrize("n_layers,hidden,inter,n_heads,n_kv,ctas", [
    (2, 2560, 9728, 32, 8, 148),           # the 2560 / 9728 block
    (3, 5120, 25600, 64, 8, 148),          # the 5120 / 25600 block (8 q heads per kv head)
    (2, 640, 1000, 4, 4, 148),             # ragged tiles, one q head per kv head
    (1, 1024, 2816, 8, 2, 16),             # the fewest CTAs the step takes
])
def test_plan_covers_every_unit_once(n_layers, hidden, inter, n_heads, n_kv, ctas):
    lib = persist._lib()
    m, layers, shapes = fake_model(n_layers, hidden, inter, n_heads, n_kv)
    size = lib.rvq_persist_plan_for(ctypes.byref(m), layers, ctas, None, 0)
    assert size > HEAD_BYTES, size
    buf = (ctypes.c_char * size)()
    assert lib.rvq_persist_plan_for(ctypes.byref(m), layers, ctas, buf, size) == size
    raw = bytes(buf)
    assert raw[:184] == bytes(m)                       # the model, as given
    n_ctas, hid_tiles, o_tiles, inter_tiles = struct.unpack_from("<4i", raw, 184)
    offs = struct.unpack_from("<5q", raw, 200)
    assert n_ctas == ctas
    tiles = lambda c: (c + 255) // 256
    assert (hid_tiles, o_tiles, inter_tiles) == (tiles(hidden), tiles(n_heads * 128), tiles(inter))
    assert list(offs) == sorted(offs) and all(o % 16 == 0 and HEAD_BYTES <= o <= size for o in offs)
    _, cf_off, jt_off, r0_off, r1_off = offs
    n_units = (r0_off - jt_off) // 4                 # up to 3 words of alignment padding
    cta_first = np.frombuffer(raw, dtype=np.int32, count=(jt_off - cf_off) // 4, offset=cf_off)
    jt = np.frombuffer(raw, dtype=np.uint32, count=n_units, offset=jt_off)
    r0 = np.frombuffer(raw, dtype=np.int32, count=n_units, offset=r0_off)
    r1 = np.frombuffer(raw, dtype=np.int32, count=n_units, offset=r1_off)
    done = 0
    for l in range(n_layers):
        for p, projs in enumerate(PHASE_JOBS):
            k = (l * 4 + p) * (ctas + 1)
            bounds = cta_first[k:k + ctas + 1]
            assert bounds[0] == done and np.all(np.diff(bounds) >= 0)
            covered = {}
            for u in range(bounds[0], bounds[-1]):
                j, t = int(jt[u]) >> 24, int(jt[u]) & 0xFFFFFF
                rows, cols = shapes[projs[j]]
                assert j < len(projs) and t < tiles(cols) and 0 <= r0[u] < r1[u] <= rows, (l, p, u)
                covered.setdefault((j, t), []).append((int(r0[u]), int(r1[u])))
            for j, pj in enumerate(projs):
                rows, cols = shapes[pj]
                for t in range(tiles(cols)):
                    spans = sorted(covered.pop((j, t)))
                    assert spans[0][0] == 0 and spans[-1][1] == rows
                    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:])), (l, p, j, t)
            assert not covered
            done = bounds[-1]
    assert 0 <= n_units - done <= 3 and r0_off - jt_off == (4 * done + 15) // 16 * 16


def test_plan_rejects_what_the_step_cannot_run():
    lib = persist._lib()
    bad = []
    m, layers, _ = fake_model(1, 1024, 2816, 8, 2)
    m.head_dim = 64
    bad.append((m, layers, _native.RVQ_ERR_UNSUPPORTED))
    m, layers, _ = fake_model(1, 1024, 2816, 32, 2)          # 16 q heads per kv head
    bad.append((m, layers, _native.RVQ_ERR_UNSUPPORTED))
    m, layers, _ = fake_model(1, 1024, 2816, 16, 2, max_len=2048)   # 8 x 2048 scores
    bad.append((m, layers, _native.RVQ_ERR_TOO_LARGE))
    m, layers, _ = fake_model(1, 1024, 2816, 8, 2)
    m.sync = 0x7000_0008                                       # not 16-byte aligned
    bad.append((m, layers, _native.RVQ_ERR_INVALID))
    m, layers, _ = fake_model(1, 1024, 2816, 8, 2)
    layers[0].proj[6].d = 4
    bad.append((m, layers, _native.RVQ_ERR_UNSUPPORTED))
    m, layers, _ = fake_model(1, 1024, 2816, 8, 2)
    layers[0].k_cache = None
    bad.append((m, layers, _native.RVQ_ERR_INVALID))
    for m, layers, status in bad:
        assert lib.rvq_persist_plan_for(ctypes.byref(m), layers, 148, None, 0) == -status
    m, layers, _ = fake_model(1, 1024, 2816, 8, 2)
    assert lib.rvq_persist_plan_for(ctypes.byref(m), layers, 8, None, 0) == -_native.RVQ_ERR_INVALID
