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


# ---------------------------------------------------------------------------
# Small batches and prompts: rvq_gemv_batch, weight-stationary tcgen05
# ---------------------------------------------------------------------------

class RvqGemvBatchJob(ctypes.Structure):
    _fields_ = [("weight", _native.RvqEntry), ("x", ctypes.c_void_p), ("y", ctypes.c_void_p),
                ("rows", ctypes.c_int64), ("cols", ctypes.c_int64), ("tokens", ctypes.c_int64),
                ("x_kind", ctypes.c_int32), ("y_kind", ctypes.c_int32), ("exact", ctypes.c_int32),
                ("reserved", ctypes.c_int32)]


_batch_bound = False


def _batch_lib():
    global _batch_bound
    lib = _native.load()
    if not _batch_bound:
        lib.rvq_gemv_batch_workspace_size.restype = ctypes.c_size_t
        lib.rvq_gemv_batch_workspace_size.argtypes = [ctypes.POINTER(RvqGemvBatchJob)]
        lib.rvq_gemv_batch.restype = ctypes.c_int
        lib.rvq_gemv_batch.argtypes = [ctypes.POINTER(RvqGemvBatchJob), ctypes.c_void_p, ctypes.c_size_t,
                                       ctypes.c_void_p]
        lib.rvq_take_batch_timeout.restype = ctypes.c_int
        lib.rvq_take_batch_timeout.argtypes = []
        _batch_bound = True
    return lib


def take_batch_timeout() -> bool:
    """Whether a bounded mbarrier wait of ``rvq_gemv_batch`` gave up since the last call."""
    v = _batch_lib().rvq_take_batch_timeout()
    if v < 0:
        _native.check(-v, "rvq_take_batch_timeout")
    return bool(v)


class BatchGemvPlan:
    """``y = x @ W^T`` for ``tokens`` bf16 rows of x (any number; blocks of at most 192)
    with W decoded on chip into the tensor cores' operand (``rvq_gemv_batch``); fixed pointers,
    so a launch can be captured in a CUDA graph.  ``entry["codes_tiled"]``
    (from ``gemv.tile_codes``) is required.  ``exact``: weights bit-identical
    to the decoded bf16 slot (slower); otherwise the stage codewords are
    summed in fp16.  The workspace (split-K partials and zeroed tickets) is
    allocated here once."""

    def __init__(self, entry: Dict[str, object], codebook: torch.Tensor, x: torch.Tensor, y: torch.Tensor,
                 exact: bool = False):
        if not gemv_supported(entry) or entry.get("codes_tiled") is None:
            raise NotImplementedError("rvq_gemv_batch needs a K=4 uint8 entry with codes_tiled")
        rows, cols = (int(s) for s in entry["shape"])
        if x.dtype != torch.bfloat16 or y.dtype != torch.bfloat16 or x.dim() != 2 or y.dim() != 2:
            raise ValueError("x [tokens, cols] and y [tokens, rows] must be bf16 matrices")
        if x.shape[1] != cols or y.shape[1] != rows or x.shape[0] != y.shape[0]:
            raise ValueError("shapes do not match the weight")
        if not x.is_contiguous() or not y.is_contiguous():
            raise ValueError("x and y must be contiguous")
        if codebook.dtype not in (torch.float16, torch.float32, torch.bfloat16):
            codebook = codebook.to(torch.float32)
        cb = codebook.contiguous()
        scales = entry["scales"].contiguous()
        codes = entry["codes_tiled"]
        w = _native.make_entry(entry["indices"], cb, scales, None, y.view(-1), d=8,
                               group_size=int(entry["group_size"]), trimmed=int(entry["trimmed_numel"]))
        w.indices = codes.data_ptr()
        self.job = RvqGemvBatchJob(w, x.data_ptr(), y.data_ptr(), rows, cols, int(x.shape[0]),
                                   _native.RVQ_BF16, _native.RVQ_BF16, 1 if exact else 0, 0)
        self.device = y.device
        with torch.cuda.device(self.device):
            nbytes = int(_batch_lib().rvq_gemv_batch_workspace_size(ctypes.byref(self.job)))
        if nbytes == 0:
            raise NotImplementedError("rvq_gemv_batch does not take this job")
        self.workspace = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
        self._keep = (cb, scales, codes, x, y)

    def launch(self, stream: Optional[int] = None) -> None:
        if stream is None:
            stream = torch.cuda.current_stream(self.device).cuda_stream
        rc = _batch_lib().rvq_gemv_batch(ctypes.byref(self.job), ctypes.c_void_p(self.workspace.data_ptr()),
                                         self.workspace.numel(), ctypes.c_void_p(stream))
        if rc:
            _native.check(rc, "rvq_gemv_batch")


def rvq_linear_batch(x: torch.Tensor, entry: Dict[str, object], codebook: torch.Tensor,
                     out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``F.linear(x, W)`` for rows of bf16 x, W decoded on chip."""
    rows = int(entry["shape"][0])
    x2 = x.reshape(-1, x.shape[-1]).contiguous()
    if out is None:
        out = torch.empty(x2.shape[0], rows, dtype=torch.bfloat16, device=x.device)
    BatchGemvPlan(entry, codebook, x2, out).launch()
    return out.view(*x.shape[:-1], rows)
