"""Oracle package: CPU restatements of the reference's RVQ reconstruction.

TEST INFRASTRUCTURE ONLY -- imported by ``tests/``, ``__graft_entry__.smoke()``
and the CPU-baseline leg of ``bench.py``; never by the ``rvq_b200`` product.

* ``rvq_oracle``      numpy restatement (the checker used by tests).
* ``rvq_oracle.c``    C/OpenMP restatement, loaded here through ctypes; it is
                      both a second checker and the timed CPU baseline.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

_HERE = os.path.dirname(os.path.abspath(__file__))
_SRC = os.path.join(_HERE, "rvq_oracle.c")
_BUILD_DIR = os.path.join(_HERE, "_build")
_LIB = os.path.join(_BUILD_DIR, "librvq_oracle.so")

_lib = None


def build_c_oracle(force: bool = False) -> str:
    """Compile ``rvq_oracle.c`` into ``oracle/_build/librvq_oracle.so``.

    Portable flags (no -march=native) so the library built here also runs on
    another x86-64 host; -ffp-contract=off keeps every add and multiply
    separately rounded.
    """
    os.makedirs(_BUILD_DIR, exist_ok=True)
    if not force and os.path.exists(_LIB) and os.path.getmtime(_LIB) >= os.path.getmtime(_SRC):
        return _LIB
    cmd = ["gcc", "-O3", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off",
           "-fno-fast-math", "-std=c11", _SRC, "-o", _LIB]
    subprocess.run(cmd, check=True)
    return _LIB


def load_c_oracle():
    global _lib
    if _lib is not None:
        return _lib
    path = build_c_oracle()
    lib = ctypes.CDLL(path)
    i64, i32, vp = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p
    lib.rvq_oracle_decode.restype = i32
    lib.rvq_oracle_decode.argtypes = [vp, i32, i64, i32, i64, vp, i32, i32, vp, i64, i64,
                                      vp, i64, vp, i32, i32]
    lib.rvq_oracle_max_threads.restype = i32
    lib.rvq_oracle_max_threads.argtypes = []
    for name in ("rvq_oracle_f32_to_f16", "rvq_oracle_f32_to_bf16"):
        fn = getattr(lib, name)
        fn.restype = None
        fn.argtypes = [vp, vp, i64]
    _lib = lib
    return lib
