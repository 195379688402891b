"""Drop-in replacement for the reference module ``triton_decode_kernels``.

Same public names, argument meaning, return value and exception types as
triton_decode_kernels.py:31-197, so the layerwise engines that import it
(infer_compressed_layerwise_triton.py:41,
infer_compressed_layerwise_single_slot.py:71-80) run unchanged.  The names
keep the word "triton" only because the engines import them by those names:
behind them is the sm_100a CUDA library (``librvq_b200.so``), one kernel
launch per call on the current torch stream, and no Triton and no CPU path.
"""

from __future__ import annotations

from typing import Dict

import torch

from . import _native

_AVAILABLE = None


def triton_available() -> bool:
    """True when the CUDA library loads and an sm_100 device is present
    (reference: triton_decode_kernels.py:31-32)."""
    global _AVAILABLE
    if _AVAILABLE is None:
        _AVAILABLE = _native.available()
    return _AVAILABLE


def rvq_triton_supported(entry: Dict[str, object], out: torch.Tensor) -> bool:
    """Reference: triton_decode_kernels.py:35-44."""
    if not triton_available():
        return False
    if not out.is_cuda:
        return False
    if int(entry["d"]) != 8:
        return False
    if entry["method"] not in ("rvq_groupwise", "rvq_mlp"):
        return False
    return True


def _device_codebook(codebook: torch.Tensor) -> torch.Tensor:
    # fp16 and fp32 codebooks are read as they are; any other float dtype is
    # widened to fp32 as the reference does (triton_decode_kernels.py:150-151).
    if codebook.dtype not in (torch.float16, torch.float32):
        codebook = codebook.to(dtype=torch.float32)
    if not codebook.is_contiguous() or codebook.data_ptr() % 16:
        codebook = codebook.contiguous().clone()
    return codebook


def _device_indices(indices: torch.Tensor) -> torch.Tensor:
    if indices.dtype not in (torch.uint8, torch.int16):
        indices = indices.to(torch.int16)
    if not indices.is_contiguous():
        indices = indices.contiguous()
    return indices


def _device_scales(scales: torch.Tensor) -> torch.Tensor:
    if scales.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        scales = scales.to(torch.float32)
    if not scales.is_contiguous():
        scales = scales.contiguous()
    return scales


def prepare_entry(entry: Dict[str, object], codebook: torch.Tensor, out: torch.Tensor):
    """Validate like decode_rvq_triton_into (triton_decode_kernels.py:119-165)
    and return the C struct for ``out``.  Raises the reference's exceptions."""
    if not triton_available():
        raise RuntimeError("Triton is not available.")

    d = int(entry["d"])
    group_size = int(entry["group_size"])
    trimmed = int(entry["trimmed_numel"])

    if d != 8:
        raise NotImplementedError(f"Triton RVQ decode currently expects d=8, got d={d}.")
    if group_size % d != 0:
        raise ValueError(f"group_size={group_size} must be divisible by d={d}.")
    if not out.is_cuda:
        raise ValueError("Triton RVQ decode requires a CUDA output tensor.")
    if not out.is_contiguous():
        raise ValueError("Triton RVQ decode requires a contiguous output tensor.")

    indices = entry["indices"]
    scales = entry["scales"]
    tail = entry["tail"]

    if not indices.is_cuda:
        raise ValueError("Triton RVQ decode requires CUDA indices.")
    if not scales.is_cuda:
        raise ValueError("Triton RVQ decode requires CUDA scales.")
    if not codebook.is_cuda:
        raise ValueError("Triton RVQ decode requires a CUDA codebook.")

    if out.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise NotImplementedError(f"Unsupported Triton RVQ output dtype: {out.dtype}")

    indices = _device_indices(indices)
    scales = _device_scales(scales)
    codebook = _device_codebook(codebook)
    if tail.numel() and tail.device != out.device:
        tail = tail.to(out.device)
    if tail.numel() and not tail.is_contiguous():
        tail = tail.contiguous()

    stages, nvec = int(indices.shape[0]), int(indices.shape[1])
    if codebook.dim() != 3 or int(codebook.shape[2]) != d or int(codebook.shape[0]) < stages:
        raise ValueError(f"codebook shape {tuple(codebook.shape)} does not match "
                         f"{stages} stages of d={d}")
    gv = group_size // d
    if nvec and scales.numel() < (nvec + gv - 1) // gv:
        raise ValueError("fewer scales than groups")
    if trimmed > nvec * d or trimmed < 0:
        raise ValueError(f"trimmed_numel={trimmed} exceeds {nvec} vectors of d={d}")
    if out.numel() < trimmed + tail.numel():
        raise ValueError("output tensor is smaller than trimmed_numel + tail")

    flat_out = out.view(-1)
    st = _native.make_entry(indices, codebook, scales, tail, flat_out, d=d,
                            group_size=group_size, trimmed=trimmed)
    # keep converted temporaries alive until the launch is queued
    return st, (indices, scales, codebook, tail)


def decode_rvq_triton_into(
    entry: Dict[str, object],
    codebook: torch.Tensor,
    out: torch.Tensor,
) -> torch.Tensor:
    """Decode ``entry`` into ``out`` on the current stream and return ``out``
    (reference: triton_decode_kernels.py:114-190)."""
    st, keep = prepare_entry(entry, codebook, out)
    dev = out.device
    if torch.cuda.current_device() != dev.index:
        with torch.cuda.device(dev):
            _native.decode(st, _native.stream_handle(dev))
    else:
        _native.decode(st, _native.stream_handle(dev))
    del keep
    return out


__all__ = [
    "decode_rvq_triton_into",
    "rvq_triton_supported",
    "triton_available",
]
