"""Tensor-parallel sharding of RVQ artifact entries (config-4 layout).

The reference runs on one GPU; tensor parallelism is new in this build.  A
Qwen3 layer is split Megatron-style across ``tp`` ranks:

* column-parallel q / k / v / gate / up: rank r keeps output rows
  ``[r * rows / tp, (r + 1) * rows / tp)`` -- whole heads for q/k/v;
* row-parallel o / down: rank r keeps input columns
  ``[r * cols / tp, (r + 1) * cols / tp)``; the ranks' products are summed by an
  all-reduce (the only exchange of the layer besides none for attention,
  which is head-local).

An RVQ entry codes 8 consecutive input elements per vector, row-major, with
one scale per ``group_size`` flattened elements (compress_full_model.py:
375-388).  A row shard is a contiguous slice of the vectors and scales; a
column shard gathers ``cols / (8 tp)`` vectors per row.  Scales must not
straddle a shard boundary: ``group_size`` has to divide the shard's row
length (row shards: any whole number of rows is fine when ``group_size``
divides ``cols``).  Entries carry no tail (the GEMV paths need none).
Sharding is exact: the shard's reconstructed weight is the same slice of
the full reconstruction, value for value.
"""

from __future__ import annotations

from typing import Dict, List, Tuple

import torch

COLUMN_PARALLEL = ("self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
                   "mlp.gate_proj.weight", "mlp.up_proj.weight")
ROW_PARALLEL = ("self_attn.o_proj.weight", "mlp.down_proj.weight")


def _check(entry: Dict[str, object]) -> Tuple[int, int, int, int]:
    if entry["method"] not in ("rvq_groupwise", "rvq_mlp"):
        raise ValueError("only RVQ entries are sharded")
    rows, cols = (int(s) for s in entry["shape"])
    d, gs = int(entry["d"]), int(entry["group_size"])
    if entry["tail"].numel() != 0 or int(entry["trimmed_numel"]) != rows * cols:
        raise NotImplementedError("sharding needs an entry without a tail")
    if cols % d:
        raise NotImplementedError("rows must hold whole vectors")
    return rows, cols, d, gs


def shard_rows(entry: Dict[str, object], rank: int, tp: int) -> Dict[str, object]:
    """Output rows ``[rank * rows / tp, (rank + 1) * rows / tp)`` of an entry."""
    rows, cols, d, gs = _check(entry)
    if rows % tp:
        raise ValueError(f"{rows} rows do not split into {tp} shards")
    rs = rows // tp
    G = cols // d
    if (rs * cols) % gs:
        raise ValueError("a scale group would straddle the row shard boundary")
    v0, v1 = rank * rs * G, (rank + 1) * rs * G
    s0, s1 = rank * rs * cols // gs, (rank + 1) * rs * cols // gs
    out = dict(entry)
    out["shape"] = [rs, cols]
    out["trimmed_numel"] = rs * cols
    out["indices"] = entry["indices"][:, v0:v1].contiguous()
    out["scales"] = entry["scales"][s0:s1].contiguous()
    out["tail"] = entry["tail"][:0].clone()
    return out


def shard_cols(entry: Dict[str, object], rank: int, tp: int) -> Dict[str, object]:
    """Input columns ``[rank * cols / tp, (rank + 1) * cols / tp)`` of an entry."""
    rows, cols, d, gs = _check(entry)
    if cols % (tp * d):
        raise ValueError(f"{cols} columns do not split into {tp} shards of whole vectors")
    cs = cols // tp
    G, Gs = cols // d, cs // d
    K = int(entry["indices"].shape[0])
    idx = entry["indices"].view(K, rows, G)[:, :, rank * Gs:(rank + 1) * Gs].reshape(K, rows * Gs)
    scales = entry["scales"]
    if gs % cols == 0:
        # a scale covers gs / cols whole rows: the shard keeps every scale, each
        # now covering the same rows of the narrower matrix
        new_scales, new_gs = scales.clone(), gs // tp
    elif cols % gs == 0 and cs % gs == 0:
        per_row = cols // gs
        new_scales = scales.view(rows, per_row)[:, rank * (cs // gs):(rank + 1) * (cs // gs)].reshape(-1).contiguous()
        new_gs = gs
    else:
        raise ValueError("a scale group would straddle the column shard boundary")
    out = dict(entry)
    out["shape"] = [rows, cs]
    out["trimmed_numel"] = rows * cs
    out["indices"] = idx.contiguous()
    out["scales"] = new_scales
    out["group_size"] = int(new_gs)
    out["tail"] = entry["tail"][:0].clone()
    return out


def shard_layer(entries: Dict[str, Dict[str, object]], layer: int, rank: int, tp: int,
                prefix: str = "model.") -> Dict[str, Dict[str, object]]:
    """The rank's entries of one decoder layer (norm weights are replicated)."""
    base = f"{prefix}layers.{layer}."
    out = {}
    for key, e in entries.items():
        if not key.startswith(base):
            continue
        name = key[len(base):]
        if name in COLUMN_PARALLEL:
            out[key] = shard_rows(e, rank, tp)
        elif name in ROW_PARALLEL:
            out[key] = shard_cols(e, rank, tp)
        else:
            out[key] = e
    return out


def shard_artifact(artifact: Dict[str, object], n_layers: int, rank: int, tp: int) -> Dict[str, object]:
    """The rank's whole artifact: sharded layers, replicated embeddings / final norm."""
    entries: Dict[str, Dict[str, object]] = {}
    for key, e in artifact["entries"].items():
        if ".layers." not in key:
            entries[key] = e
    for l in range(n_layers):
        entries.update(shard_layer(artifact["entries"], l, rank, tp))
    out = dict(artifact)
    out["entries"] = entries
    return out


def sharded_dims(n_heads: int, n_kv: int, intermediate: int, tp: int) -> Tuple[int, int, int]:
    """Per-rank (query heads, kv heads, intermediate) of a tp-way split."""
    if n_heads % tp or n_kv % tp or intermediate % tp:
        raise ValueError(f"heads {n_heads}/{n_kv} and intermediate {intermediate} must split {tp} ways")
    return n_heads // tp, n_kv // tp, intermediate // tp
