"""ctypes binding of ``librvq_b200.so`` (declared in include/rvq_b200.h).

There is no fallback: if the library is missing or has no usable sm_100
device, every entry point raises.
"""

from __future__ import annotations

import ctypes
import os
from typing import Iterable, List, Optional, Sequence, Tuple

import torch

from .build import LIB_PATH

RVQ_OK = 0
RVQ_ERR_INVALID = 1
RVQ_ERR_UNSUPPORTED = 2
RVQ_ERR_UNAVAILABLE = 3
RVQ_ERR_CUDA = 4
RVQ_ERR_TOO_LARGE = 5

RVQ_F16, RVQ_BF16, RVQ_F32, RVQ_U8, RVQ_I16, RVQ_U8X4 = 0, 1, 2, 3, 4, 5
RVQ_MAX_LAYER_JOBS = 32

KIND_OF_DTYPE = {
    torch.float16: RVQ_F16,
    torch.bfloat16: RVQ_BF16,
    torch.float32: RVQ_F32,
    torch.uint8: RVQ_U8,
    torch.int16: RVQ_I16,
}

EXPORTED_SYMBOLS = (
    "rvq_available", "rvq_check_entry", "rvq_decode", "rvq_decode_layer", "rvq_decode_int8",
    "rvq_check_int8_entry", "rvq_decode_layer_mixed",
    "rvq_take_index_error", "rvq_last_cuda_error", "rvq_status_string", "rvq_version",
)


class RvqEntry(ctypes.Structure):
    _fields_ = [
        ("indices", ctypes.c_void_p),
        ("codebook", ctypes.c_void_p),
        ("scales", ctypes.c_void_p),
        ("tail", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("nvec", ctypes.c_int64),
        ("stage_stride", ctypes.c_int64),
        ("group_vecs", ctypes.c_int64),
        ("trimmed", ctypes.c_int64),
        ("tail_numel", ctypes.c_int64),
        ("stages", ctypes.c_int32),
        ("ncodes", ctypes.c_int32),
        ("d", ctypes.c_int32),
        ("index_kind", ctypes.c_int32),
        ("codebook_kind", ctypes.c_int32),
        ("scale_kind", ctypes.c_int32),
        ("tail_kind", ctypes.c_int32),
        ("out_kind", ctypes.c_int32),
    ]


class RvqCopy(ctypes.Structure):
    _fields_ = [
        ("src", ctypes.c_void_p),
        ("dst", ctypes.c_void_p),
        ("nbytes", ctypes.c_int64),
    ]


class RvqInt8Entry(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p),
        ("scales", ctypes.c_void_p),
        ("tail", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("trimmed", ctypes.c_int64),
        ("group_size", ctypes.c_int64),
        ("tail_numel", ctypes.c_int64),
        ("scale_kind", ctypes.c_int32),
        ("tail_kind", ctypes.c_int32),
        ("out_kind", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


class RvqError(RuntimeError):
    def __init__(self, status: int, where: str, message: str):
        super().__init__(f"{where}: {message} (status {status})")
        self.status = status


_lib = None


def library_path() -> str:
    return LIB_PATH


def load() -> ctypes.CDLL:
    """Load the CUDA library; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"rvq_b200 CUDA library not found at {LIB_PATH}; build it with "
            "`python -m rvq_b200.build` (nvcc, sm_100a)")
    lib = ctypes.CDLL(LIB_PATH)
    vp, i32 = ctypes.c_void_p, ctypes.c_int
    lib.rvq_available.restype = i32
    lib.rvq_available.argtypes = []
    lib.rvq_check_entry.restype = i32
    lib.rvq_check_entry.argtypes = [ctypes.POINTER(RvqEntry)]
    lib.rvq_decode.restype = i32
    lib.rvq_decode.argtypes = [ctypes.POINTER(RvqEntry), vp]
    lib.rvq_decode_layer.restype = i32
    lib.rvq_decode_layer.argtypes = [ctypes.POINTER(RvqEntry), i32, ctypes.POINTER(RvqCopy), i32, vp]
    lib.rvq_check_int8_entry.restype = i32
    lib.rvq_check_int8_entry.argtypes = [ctypes.POINTER(RvqInt8Entry)]
    lib.rvq_decode_int8.restype = i32
    lib.rvq_decode_int8.argtypes = [ctypes.POINTER(RvqInt8Entry), vp]
    lib.rvq_decode_layer_mixed.restype = i32
    lib.rvq_decode_layer_mixed.argtypes = [ctypes.POINTER(RvqEntry), i32, ctypes.POINTER(RvqInt8Entry), i32,
                                           ctypes.POINTER(RvqCopy), i32, vp]
    lib.rvq_decode_layer_ctas.restype = i32
    lib.rvq_decode_layer_ctas.argtypes = [ctypes.POINTER(RvqEntry), i32, ctypes.POINTER(RvqInt8Entry), i32,
                                          ctypes.POINTER(RvqCopy), i32, i32, vp]
    lib.rvq_take_index_error.restype = i32
    lib.rvq_take_index_error.argtypes = []
    lib.rvq_last_cuda_error.restype = i32
    lib.rvq_last_cuda_error.argtypes = []
    lib.rvq_status_string.restype = ctypes.c_char_p
    lib.rvq_status_string.argtypes = [i32]
    lib.rvq_version.restype = i32
    lib.rvq_version.argtypes = []
    lib.rvq_test_fastdiv.restype = ctypes.c_uint32
    lib.rvq_test_fastdiv.argtypes = [ctypes.c_uint32, ctypes.c_uint32]
    _lib = lib
    return lib


def status_string(status: int) -> str:
    return load().rvq_status_string(int(status)).decode()


def check(status: int, where: str) -> None:
    if status == RVQ_OK:
        return
    msg = status_string(status)
    if status == RVQ_ERR_CUDA:
        msg += f" (cudaError {load().rvq_last_cuda_error()})"
    raise RvqError(status, where, msg)


def available() -> bool:
    if not torch.cuda.is_available():
        return False
    return bool(load().rvq_available())


def kind_of(t: torch.Tensor) -> int:
    try:
        return KIND_OF_DTYPE[t.dtype]
    except KeyError:
        raise NotImplementedError(f"unsupported dtype {t.dtype}") from None


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def make_entry(indices: torch.Tensor, codebook: torch.Tensor, scales: torch.Tensor,
               tail: Optional[torch.Tensor], out_flat: torch.Tensor, *, d: int,
               group_size: int, trimmed: int) -> RvqEntry:
    """Fill the C struct from device tensors (no copies, no checks beyond
    what the struct needs; the library validates the rest)."""
    e = RvqEntry()
    stages, nvec = int(indices.shape[0]), int(indices.shape[1])
    e.indices = indices.data_ptr() if indices.numel() else None
    e.codebook = codebook.data_ptr() if codebook.numel() else None
    e.scales = scales.data_ptr() if scales.numel() else None
    tail_n = int(tail.numel()) if tail is not None else 0
    e.tail = tail.data_ptr() if tail_n else None
    e.out = out_flat.data_ptr()
    e.nvec = nvec
    e.stage_stride = int(indices.stride(0)) if stages > 1 else nvec
    e.group_vecs = int(group_size) // int(d)
    e.trimmed = int(trimmed)
    e.tail_numel = tail_n
    e.stages = stages
    e.ncodes = int(codebook.shape[1])
    e.d = int(d)
    e.index_kind = kind_of(indices)
    e.codebook_kind = kind_of(codebook)
    e.scale_kind = kind_of(scales)
    e.tail_kind = kind_of(tail) if tail_n else RVQ_BF16
    e.out_kind = kind_of(out_flat)
    return e


def make_int8_entry(q: torch.Tensor, scales: torch.Tensor, tail: Optional[torch.Tensor],
                    out_flat: torch.Tensor, *, group_size: int, trimmed: int) -> RvqInt8Entry:
    """The C struct of an int8_groupwise entry from device tensors (q int8,
    contiguous; the library validates sizes and kinds)."""
    e = RvqInt8Entry()
    e.q = q.data_ptr() if q.numel() else None
    e.scales = scales.data_ptr() if scales.numel() else None
    tail_n = int(tail.numel()) if tail is not None else 0
    e.tail = tail.data_ptr() if tail_n else None
    e.out = out_flat.data_ptr()
    e.trimmed = int(trimmed)
    e.group_size = int(group_size)
    e.tail_numel = tail_n
    e.scale_kind = kind_of(scales)
    e.tail_kind = kind_of(tail) if tail_n else RVQ_BF16
    e.out_kind = kind_of(out_flat)
    return e


def decode(entry: RvqEntry, stream: int) -> None:
    check(load().rvq_decode(ctypes.byref(entry), ctypes.c_void_p(stream)), "rvq_decode")


def decode_layer(entries: Sequence[RvqEntry], copies: Sequence[Tuple[int, int, int]],
                 stream: int) -> None:
    n, m = len(entries), len(copies)
    if n + m > RVQ_MAX_LAYER_JOBS:
        raise ValueError(f"at most {RVQ_MAX_LAYER_JOBS} entries + copies per layer launch")
    arr = (RvqEntry * max(n, 1))(*entries)
    carr = (RvqCopy * max(m, 1))(*[RvqCopy(s, d, b) for (s, d, b) in copies])
    check(load().rvq_decode_layer(arr, n, carr, m, ctypes.c_void_p(stream)), "rvq_decode_layer")


def take_index_error() -> bool:
    r = load().rvq_take_index_error()
    if r < 0:
        check(-r, "rvq_take_index_error")
    return bool(r)
