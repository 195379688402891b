"""Prefill GEMM with the RVQ weight decoded into shared memory
(``rvq_gemm_prefill``, include/rvq_b200.h): ``y = x @ W^T`` for a prompt of
``m`` tokens on tcgen05 tensor cores, W never written to HBM.  The
reference's prefill is decode-into-slot + ``F.linear``
(infer_compressed_layerwise_triton.py:263, 290-292).
"""

from __future__ import annotations

import ctypes
from typing import Dict, Optional

import torch

from . import _native
from .gemv import gemv_supported

_bound = False


class RvqGemmJob(ctypes.Structure):
    _fields_ = [("weight", _native.RvqEntry), ("x", ctypes.c_void_p), ("y", ctypes.c_void_p),
                ("m", ctypes.c_int64), ("n", ctypes.c_int64), ("k", ctypes.c_int64),
                ("x_kind", ctypes.c_int32), ("y_kind", ctypes.c_int32)]


def _lib():
    global _bound
    lib = _native.load()
    if not _bound:
        lib.rvq_gemm_prefill.restype = ctypes.c_int
        lib.rvq_gemm_prefill.argtypes = [ctypes.POINTER(RvqGemmJob), ctypes.c_void_p]
        lib.rvq_take_gemm_timeout.restype = ctypes.c_int
        lib.rvq_take_gemm_timeout.argtypes = []
        _bound = True
    return lib


def take_timeout() -> bool:
    """Whether a bounded mbarrier wait of a prefill GEMM gave up since the last call."""
    v = _lib().rvq_take_gemm_timeout()
    if v < 0:
        _native.check(-v, "rvq_take_gemm_timeout")
    return bool(v)


class GemmPlan:
    """One ``rvq_gemm_prefill`` call with fixed pointers (graph-capturable).
    ``entry["codes_il"]`` (from ``gemv.interleave_codes``) is required."""

    def __init__(self, entry: Dict[str, object], codebook: torch.Tensor, x: torch.Tensor, y: torch.Tensor):
        if not gemv_supported(entry) or entry.get("codes_il") is None:
            raise NotImplementedError("rvq_gemm_prefill needs a K=4 uint8 entry with codes_il")
        n, k = (int(s) for s in entry["shape"])
        if x.dtype != torch.bfloat16 or y.dtype != torch.bfloat16 or x.dim() != 2 or y.dim() != 2:
            raise ValueError("x [m, k] and y [m, n] must be bf16 matrices")
        if x.shape[1] != k or y.shape[1] != n or x.shape[0] != y.shape[0]:
            raise ValueError("shapes do not match the weight")
        if not x.is_contiguous() or not y.is_contiguous():
            raise ValueError("x and y must be contiguous")
        cb = codebook.to(torch.float32).contiguous()
        scales = entry["scales"].contiguous()
        codes = entry["codes_il"]
        w = _native.make_entry(entry["indices"], cb, scales, None, y.view(-1), d=8,
                               group_size=int(entry["group_size"]), trimmed=int(entry["trimmed_numel"]))
        w.indices = codes.data_ptr()
        self._keep = (cb, scales, codes, x, y)
        self.job = RvqGemmJob(w, x.data_ptr(), y.data_ptr(), int(x.shape[0]), n, k, _native.RVQ_BF16, _native.RVQ_BF16)
        self.device = y.device

    def launch(self, stream: Optional[int] = None) -> None:
        if stream is None:
            stream = torch.cuda.current_stream(self.device).cuda_stream
        rc = _lib().rvq_gemm_prefill(ctypes.byref(self.job), ctypes.c_void_p(stream))
        if rc:
            _native.check(rc, "rvq_gemm_prefill")


def rvq_matmul(x: torch.Tensor, entry: Dict[str, object], codebook: torch.Tensor,
               out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``F.linear(x, W)`` for a [m, k] bf16 prompt, W decoded on chip."""
    n = int(entry["shape"][0])
    x2 = x.reshape(-1, x.shape[-1]).contiguous()
    if out is None:
        out = torch.empty(x2.shape[0], n, dtype=torch.bfloat16, device=x.device)
    GemmPlan(entry, codebook, x2, out).launch()
    return out.view(*x.shape[:-1], n)
