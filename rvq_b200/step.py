"""Python binding of the batch-1 decode-step operations (include/rvq_b200.h:
``rvq_step_norm``, ``rvq_step_attention``, ``rvq_step_silu_mul``).

Each ``*Op`` resolves its pointers once; ``launch()`` queues one kernel on
the current stream, so a sequence of ops can be captured in a CUDA graph.
The tensors an op was built from must outlive it and keep their storage.
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _native


class RvqVec(ctypes.Structure):
    _fields_ = [("ptr", ctypes.c_void_p), ("n", ctypes.c_int64), ("ntiles", ctypes.c_int32),
                ("kind", ctypes.c_int32)]


class RvqNormArgs(ctypes.Structure):
    _fields_ = [("h", ctypes.c_void_p), ("add", RvqVec), ("token", ctypes.c_void_p),
                ("embed", ctypes.c_void_p), ("weight", ctypes.c_void_p), ("x", ctypes.c_void_p),
                ("hidden", ctypes.c_int64), ("eps", ctypes.c_float), ("vocab", ctypes.c_int32),
                ("arrivals", ctypes.c_void_p), ("consumed", ctypes.c_void_p),
                ("arrivals_per_use", ctypes.c_uint32), ("reserved", ctypes.c_int32)]


class RvqAttnArgs(ctypes.Structure):
    _fields_ = [("q", RvqVec), ("k", RvqVec), ("v", RvqVec),
                ("q_norm", ctypes.c_void_p), ("k_norm", ctypes.c_void_p),
                ("cos", ctypes.c_void_p), ("sin", ctypes.c_void_p), ("pos", ctypes.c_void_p),
                ("k_cache", ctypes.c_void_p), ("v_cache", ctypes.c_void_p), ("out", ctypes.c_void_p),
                ("n_heads", ctypes.c_int32), ("n_kv", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("max_len", ctypes.c_int32), ("eps", ctypes.c_float), ("scaling", ctypes.c_float),
                ("valid_bias", ctypes.c_float), ("reserved", ctypes.c_int32)]


_bound = False


def _lib():
    global _bound
    lib = _native.load()
    if not _bound:
        lib.rvq_step_norm.restype = ctypes.c_int
        lib.rvq_step_norm.argtypes = [ctypes.POINTER(RvqNormArgs), ctypes.c_void_p]
        lib.rvq_step_attention.restype = ctypes.c_int
        lib.rvq_step_attention.argtypes = [ctypes.POINTER(RvqAttnArgs), ctypes.c_void_p]
        lib.rvq_step_silu_mul.restype = ctypes.c_int
        lib.rvq_step_silu_mul.argtypes = [ctypes.POINTER(RvqVec), ctypes.POINTER(RvqVec), ctypes.c_void_p,
                                          ctypes.c_void_p]
        _bound = True
    return lib


def _bf16(t: torch.Tensor, name: str) -> int:
    if t.dtype != torch.bfloat16 or not t.is_cuda or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous CUDA bf16 tensor")
    return t.data_ptr()


def vec(t: Optional[torch.Tensor], ntiles: int = 1) -> RvqVec:
    """A vector operand: a bf16/fp16 vector, or fp32 partials [ntiles, n]."""
    if t is None:
        return RvqVec(None, 0, 0, 0)
    if not t.is_cuda or not t.is_contiguous():
        raise ValueError("vector operands are contiguous CUDA tensors")
    if t.dtype == torch.float32:
        n = t.numel() // ntiles
        if n * ntiles != t.numel():
            raise ValueError("partials do not split into ntiles rows")
        return RvqVec(t.data_ptr(), n, ntiles, _native.RVQ_F32)
    if ntiles != 1:
        raise ValueError("a bf16/fp16 operand has one tile")
    return RvqVec(t.data_ptr(), t.numel(), 1, _native.kind_of(t))


def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


class NormOp:
    """``h <- h + add`` (or ``embed[token]``), ``x <- rmsnorm(h) * weight``.
    ``landing``: a tensor-parallel landing buffer (``PeerExchange.landing``)
    to wait for and add instead of ``add``."""

    def __init__(self, h, weight, x, eps, add=None, add_tiles=1, token=None, embed=None, landing=None):
        hidden = h.numel()
        if weight.numel() != hidden or x.numel() != hidden:
            raise ValueError("h, weight and x must have the same length")
        if token is not None and (token.dtype != torch.int64 or not token.is_cuda or embed is None
                                  or embed.dim() != 2 or embed.shape[1] != hidden):
            raise ValueError("token must be a CUDA int64 tensor and embed a [vocab, hidden] table")
        self._keep = (h, weight, x, add, token, embed)
        self.args = RvqNormArgs(_bf16(h, "h"), vec(add, add_tiles),
                                None if token is None else token.data_ptr(),
                                None if embed is None else _bf16(embed, "embed"),
                                _bf16(weight, "weight"), _bf16(x, "x"), hidden, float(eps),
                                0 if embed is None else int(embed.shape[0]))
        if landing is not None:
            if add is not None or token is not None:
                raise ValueError("landing replaces add and excludes token")
            self.args.add = RvqVec(landing["add"], hidden, landing["tp"], _native.RVQ_F32)
            self.args.arrivals, self.args.consumed = landing["arrivals"], landing["consumed"]
            self.args.arrivals_per_use = landing["per_use"]

    def launch(self) -> None:
        rc = _lib().rvq_step_norm(ctypes.byref(self.args), _stream())
        if rc:
            _native.check(rc, "rvq_step_norm")


class AttentionOp:
    """Decode attention of one token for one layer (see rvq_step_attention)."""

    def __init__(self, q, k, v, q_norm, k_norm, cos, sin, pos, k_cache, v_cache, out, *,
                 n_heads, n_kv, head_dim, eps, scaling, valid_bias, q_tiles=1, kv_tiles=1):
        max_len = int(cos.shape[0])
        if tuple(k_cache.shape) != (n_kv, max_len, head_dim) or k_cache.shape != v_cache.shape:
            raise ValueError("caches must be [n_kv, max_len, head_dim]")
        if pos.dtype != torch.int64 or not pos.is_cuda:
            raise ValueError("pos must be a CUDA int64 tensor")
        self._keep = (q, k, v, q_norm, k_norm, cos, sin, pos, k_cache, v_cache, out)
        self.args = RvqAttnArgs(vec(q, q_tiles), vec(k, kv_tiles), vec(v, kv_tiles),
                                _bf16(q_norm, "q_norm"), _bf16(k_norm, "k_norm"), _bf16(cos, "cos"),
                                _bf16(sin, "sin"), pos.data_ptr(), _bf16(k_cache, "k_cache"),
                                _bf16(v_cache, "v_cache"), _bf16(out, "out"), n_heads, n_kv, head_dim,
                                max_len, float(eps), float(scaling), float(valid_bias), 0)

    def launch(self) -> None:
        rc = _lib().rvq_step_attention(ctypes.byref(self.args), _stream())
        if rc:
            _native.check(rc, "rvq_step_attention")


class SiluMulOp:
    """``out = bf16(bf16(silu(gate)) * up)``."""

    def __init__(self, gate, up, out, gate_tiles=1, up_tiles=1):
        self._keep = (gate, up, out)
        self.g, self.u = vec(gate, gate_tiles), vec(up, up_tiles)
        self.out = _bf16(out, "out")

    def launch(self) -> None:
        rc = _lib().rvq_step_silu_mul(ctypes.byref(self.g), ctypes.byref(self.u), ctypes.c_void_p(self.out),
                                      _stream())
        if rc:
            _native.check(rc, "rvq_step_silu_mul")
