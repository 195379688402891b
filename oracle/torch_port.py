"""PyTorch CPU restatements of the reference's own reconstruction functions.

TEST AND BASELINE INFRASTRUCTURE ONLY -- used by ``tests/`` and by the
CPU-baseline / reference legs of ``bench.py``; never by the ``rvq_b200``
product.  The reference's engine cannot be imported where the benchmark
runs, so these restate, with the same PyTorch operations in the same order,

* ``_decode_rvq_into``  (infer_compressed_layerwise_single_slot.py:123-149):
  int64 indices, fp32 codebook, an advanced-index gather of every stage for
  a chunk of ``chunk // stages`` vectors, ``sum(dim=0)`` over the stages,
  the product with the per-group scales, and a ``copy_`` into the output
  dtype (round to nearest even);
* ``_decode_int8_into`` (same file, 110-120): ``q * scales`` per group, then
  the tail.

Timing these on the host's cores is the "reference's PyTorch
reconstruction" baseline; their outputs are also checked bit for bit against
the numpy / C oracles and the reference-produced golden vectors.
"""

from __future__ import annotations

from typing import Dict

import torch


def _f32(t: torch.Tensor) -> torch.Tensor:
    return t if t.dtype == torch.float32 else t.to(torch.float32)


def decode_rvq_into(entry: Dict[str, object], codebook: torch.Tensor, out: torch.Tensor,
                    chunk: int = 262144) -> torch.Tensor:
    """Restates infer_compressed_layerwise_single_slot.py:123-149."""
    d = int(entry["d"])
    group_size = int(entry["group_size"])
    trimmed = int(entry["trimmed_numel"])
    scales = _f32(entry["scales"])
    indices = entry["indices"]
    indices = indices if indices.dtype == torch.int64 else indices.to(torch.int64)
    tail = _f32(entry["tail"])
    codebook = _f32(codebook).contiguous()
    stages, nvec = indices.shape
    recon = torch.empty((nvec, d), dtype=torch.float32, device=codebook.device)
    stage_ids = torch.arange(stages, device=codebook.device)
    step = max(1, chunk // max(stages, 1))
    for start in range(0, nvec, step):
        end = min(start + step, nvec)
        recon[start:end].copy_(codebook[stage_ids[:, None], indices[:, start:end]].sum(dim=0))
    core = (recon.reshape(-1, group_size) * scales.unsqueeze(1)).reshape(-1)[:trimmed]
    flat = out.view(-1)
    flat[:trimmed].copy_(core)
    if tail.numel():
        flat[trimmed:trimmed + tail.numel()].copy_(tail)
    return out


def decode_int8_into(entry: Dict[str, object], out: torch.Tensor) -> torch.Tensor:
    """Restates infer_compressed_layerwise_single_slot.py:110-120."""
    q = _f32(entry["q"])
    scales = _f32(entry["scales"])
    tail = _f32(entry["tail"])
    trimmed = int(entry["trimmed_numel"])
    core = (q * scales.unsqueeze(1)).reshape(-1)[:trimmed]
    flat = out.view(-1)
    flat[:trimmed].copy_(core)
    if tail.numel():
        flat[trimmed:trimmed + tail.numel()].copy_(tail)
    return out
