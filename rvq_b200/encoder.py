"""The compressor's RVQ encoder and k-means on the GPU.

Drop-in GPU versions of compress_full_model.py's hot functions, with the same
arguments and results (tensors on the GPU instead of the CPU):

* ``assign_codes(x, c, chunk_size)``                       -- lines 202-208
* ``kmeans_train(x, k, iters, seed, chunk_size)``          -- lines 211-234
* ``encode_rvq_tensor(t, codebooks, d, group_size, chunk_size, codebook_id)``
                                                           -- lines 337-388

The distance computation and argmin run in ``rvq_kmeans_step`` /
``rvq_encode_vectors`` (rvq_b200/csrc/rvq_encode.cu); group normalisation,
the centroid division and the error statistics are a few tensor operations
around them.  ``chunk_size`` is accepted for signature compatibility (the
kernels stream the vectors themselves).

Parity: the reference sums the 8-term dot products in its CPU BLAS's order,
so where two codewords' distances differ only in the last bits the chosen
codes may differ; k-means centroid sums are accumulated in order-independent
64-bit fixed point (deterministic), the reference's in fp32 row order.
"""

from __future__ import annotations

import ctypes
import math
from typing import Dict

import torch

from . import _native

_bound = False


def _lib():
    global _bound
    lib = _native.load()
    if not _bound:
        vp, i32, i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
        lib.rvq_encode_vectors.restype = i32
        lib.rvq_encode_vectors.argtypes = [vp, i64, vp, i32, i32, i32, vp, i32, vp, vp]
        lib.rvq_kmeans_step.restype = i32
        lib.rvq_kmeans_step.argtypes = [vp, i64, vp, i32, i32, vp, vp, vp, vp]
        _bound = True
    return lib


def _stream(device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _vectors(x: torch.Tensor) -> torch.Tensor:
    if not x.is_cuda or x.dim() != 2 or x.shape[1] != 8:
        raise NotImplementedError("the GPU encoder takes CUDA [n, 8] vectors")
    return x.to(torch.float32).contiguous()


def kmeans_assign_stats(x: torch.Tensor, centroids: torch.Tensor, with_stats: bool = True):
    """Nearest centroid of every row of x (int32), and the per-centroid fixed
    point sums / counts when ``with_stats``."""
    x = _vectors(x)
    cent = centroids.to(torch.float32).contiguous()
    n, k = x.shape[0], cent.shape[0]
    assign = torch.empty(n, dtype=torch.int32, device=x.device)
    sums = torch.zeros(k, 8, dtype=torch.int64, device=x.device) if with_stats else None
    counts = torch.zeros(k, dtype=torch.int64, device=x.device) if with_stats else None
    with torch.cuda.device(x.device):
        _native.check(_lib().rvq_kmeans_step(x.data_ptr(), n, cent.data_ptr(), k, 8, assign.data_ptr(),
                                             sums.data_ptr() if with_stats else None,
                                             counts.data_ptr() if with_stats else None, _stream(x.device)),
                      "rvq_kmeans_step")
    return assign, sums, counts


def assign_codes(x: torch.Tensor, c: torch.Tensor, chunk_size: int = 65536) -> torch.Tensor:
    """compress_full_model.py:202-208 on the GPU: int64 index of the nearest codeword."""
    return kmeans_assign_stats(x, c, with_stats=False)[0].to(torch.int64)


def kmeans_train(x: torch.Tensor, k: int, iters: int, seed: int, chunk_size: int = 65536) -> torch.Tensor:
    """compress_full_model.py:211-234 on the GPU.  The same CPU generator
    draws the initial centroids and the refills of empty clusters."""
    x = _vectors(x)
    n = x.shape[0]
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    init_idx = torch.randperm(n, generator=g)[:k].to(x.device)
    centroids = x[init_idx].clone()
    for _ in range(iters):
        _, sums, counts = kmeans_assign_stats(x, centroids)
        nz = counts > 0
        mean = (sums.to(torch.float64) / 2.0 ** 32) / counts.clamp_min(1).to(torch.float64).unsqueeze(1)
        centroids[nz] = mean[nz].to(torch.float32)
        dead = (~nz).nonzero(as_tuple=False).view(-1)
        if dead.numel() > 0:
            refill = torch.randperm(n, generator=g)[: dead.numel()].to(x.device)
            centroids[dead] = x[refill]
    return centroids


def normalize_groups(flat: torch.Tensor, group_size: int, eps: float = 1e-8):
    """compress_full_model.py:237-246 (the same tensor operations)."""
    trimmed = (flat.numel() // group_size) * group_size
    core, tail = flat[:trimmed], flat[trimmed:]
    if trimmed == 0:
        return None, None, tail
    groups = core.view(-1, group_size)
    scales = groups.abs().amax(dim=1).clamp_min(eps)
    return (groups / scales.unsqueeze(1)).contiguous(), scales.contiguous(), tail.contiguous()


def encode_rvq_tensor(t: torch.Tensor, codebooks: torch.Tensor, d: int, group_size: int,
                      chunk_size: int = 65536, codebook_id: str = "") -> Dict[str, object]:
    """compress_full_model.py:337-388 on the GPU: the artifact entry of ``t``
    (tensors on the GPU)."""
    if d != 8:
        raise NotImplementedError("the GPU encoder takes d = 8")
    dev = codebooks.device if codebooks.is_cuda else t.device
    flat = t.to(dev, torch.float32).reshape(-1)
    norm, scales, tail = normalize_groups(flat, group_size)
    if norm is None:
        raise RuntimeError("Tensor too small for RVQ group size.")
    usable = (norm.numel() // d) * d
    x = norm.reshape(-1)[:usable].view(-1, d).contiguous()
    cb = codebooks.to(dev, torch.float32).contiguous()
    stages, k = int(cb.shape[0]), int(cb.shape[1])
    code_dtype = torch.uint8 if k <= 256 else torch.int16
    codes = torch.empty(stages, x.shape[0], dtype=code_dtype, device=dev)
    residual = torch.empty_like(x)
    with torch.cuda.device(dev):
        _native.check(_lib().rvq_encode_vectors(x.data_ptr(), x.shape[0], cb.data_ptr(), stages, k, d,
                                                codes.data_ptr(), _native.RVQ_U8 if k <= 256 else _native.RVQ_I16,
                                                residual.data_ptr(), _stream(dev)), "rvq_encode_vectors")
    recon = torch.zeros_like(x)                  # the chosen codewords summed in stage order, as the reference
    for r in range(stages):
        recon += cb[r][codes[r].long()]
    recon_core = (recon.reshape(-1).view(-1, group_size) * scales.unsqueeze(1)).reshape(-1)
    ref_core = flat[: recon_core.numel()]
    err = recon_core - ref_core
    mse = float((err * err).mean().item())
    denom = float(torch.sqrt((ref_core * ref_core).mean()).item()) + 1e-12
    return {
        "method": "rvq_groupwise",
        "codebook_id": codebook_id,
        "shape": list(t.shape),
        "dtype": str(t.dtype).replace("torch.", ""),
        "group_size": int(group_size),
        "d": int(d),
        "trimmed_numel": int(recon_core.numel()),
        "scales": scales.to(torch.float16),
        "indices": codes,
        "tail": tail.to(torch.bfloat16),
        "mse": mse,
        "rel_rmse": math.sqrt(mse) / denom,
    }
