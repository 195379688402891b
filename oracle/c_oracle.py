"""numpy-facing wrapper of the C oracle (``rvq_oracle.c``).

TEST INFRASTRUCTURE ONLY (tests, smoke check, CPU baseline of bench.py).
"""

from __future__ import annotations

import numpy as np

from . import load_c_oracle
from .rvq_oracle import OUT_F32, RVQEntryNP


def decode_rvq_bits_c(entry: RVQEntryNP, out_kind: int, nthreads: int = 0,
                      out: np.ndarray | None = None) -> np.ndarray:
    """Same contract as ``rvq_oracle.decode_rvq_bits`` computed by the C port."""
    lib = load_c_oracle()
    idx = np.ascontiguousarray(entry.indices)
    if idx.dtype == np.uint8:
        ib = 1
    elif idx.dtype == np.int16:
        ib = 2
    else:
        raise TypeError(f"indices dtype {idx.dtype} not supported")
    cb = np.ascontiguousarray(entry.codebook, dtype=np.float32)
    sc = np.ascontiguousarray(entry.scales, dtype=np.float32)
    tail = np.ascontiguousarray(entry.tail, dtype=np.float32)
    bits_dtype = np.uint32 if out_kind == OUT_F32 else np.uint16
    if out is None:
        out = np.zeros(int(entry.numel), dtype=bits_dtype)
    K, nvec = idx.shape
    rc = lib.rvq_oracle_decode(
        idx.ctypes.data, ib, nvec, K, nvec, cb.ctypes.data, cb.shape[1], int(entry.d),
        sc.ctypes.data, int(entry.group_size) // int(entry.d), int(entry.trimmed_numel),
        tail.ctypes.data, tail.size, out.ctypes.data, int(out_kind), int(nthreads))
    if rc == -2:
        raise IndexError("RVQ index out of range of the codebook")
    if rc != 0:
        raise ValueError(f"rvq_oracle_decode rejected its arguments (rc={rc})")
    return out


def max_threads() -> int:
    return int(load_c_oracle().rvq_oracle_max_threads())
