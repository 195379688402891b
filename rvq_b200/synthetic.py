"""Seeded synthetic RVQ artifacts in the reference's entry format.

There is no checkpoint on the GPU hosts, so every workload is generated from
a ``torch.Generator`` seed.  Entries follow the dict layout written by
``encode_rvq_tensor`` (compress_full_model.py:375-388) and the artifact layout
of compress_full_model.py:624-629; 1-D tensors are ``bf16_raw`` entries as in
compress_full_model.py:594-601.

Distributions:
* codebook stage k: N(0, (0.02 * 2**-k)**2), stored fp16 ``[K, ncodes, d]``
  (the artifact stores fp16 codebooks, compress_full_model.py:334);
* indices: uniform over ``[0, ncodes)``, uint8 when ``ncodes <= 256`` else
  int16 (compress_full_model.py:374), layout ``[K, out * in / d]``;
* scales: uniform in [0.5, 1.5], fp16, one per output row by default
  (``group_size == in_features``) or one per ``group_size`` flattened
  elements;
* norm weights: 1 + N(0, 0.02**2) in bf16.

Everything is generated on the CPU, so the same seed gives the same bytes on
any host running the same torch build.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import torch


def make_codebook(stages: int, ncodes: int, d: int, gen: torch.Generator,
                  sigma0: float = 0.02) -> torch.Tensor:
    cb = torch.empty((stages, ncodes, d), dtype=torch.float32)
    for k in range(stages):
        cb[k].normal_(0.0, sigma0 * (2.0 ** -k), generator=gen)
    return cb.to(torch.float16).contiguous()


def make_rvq_entry(out_features: int, in_features: int, gen: torch.Generator, *,
                   stages: int = 4, ncodes: int = 256, d: int = 8,
                   group_size: Optional[int] = None, codebook_id: str = "global_2d",
                   dtype: str = "bfloat16") -> Dict[str, object]:
    """One RVQ entry for a ``[out_features, in_features]`` weight.

    ``group_size=None`` means one scale per output row.  A numel that is not a
    multiple of ``group_size`` leaves a bf16 ``tail`` exactly as
    ``normalize_groups`` does (compress_full_model.py:237-246).
    """
    numel = out_features * in_features
    if group_size is None:
        group_size = in_features
    if group_size % d != 0:
        raise ValueError("group_size must be divisible by d")
    trimmed = (numel // group_size) * group_size
    nvec = trimmed // d
    tail_numel = numel - trimmed
    idx_dtype = torch.uint8 if ncodes <= 256 else torch.int16
    indices = torch.randint(0, ncodes, (stages, nvec), dtype=idx_dtype, generator=gen)
    scales = torch.empty(trimmed // group_size, dtype=torch.float32).uniform_(
        0.5, 1.5, generator=gen).to(torch.float16)
    tail = (torch.randn(tail_numel, generator=gen) * 0.02).to(torch.bfloat16)
    return {
        "method": "rvq_groupwise",
        "codebook_id": codebook_id,
        "shape": [out_features, in_features],
        "dtype": dtype,
        "group_size": int(group_size),
        "d": int(d),
        "trimmed_numel": int(trimmed),
        "scales": scales.contiguous(),
        "indices": indices.contiguous(),
        "tail": tail.contiguous(),
        "mse": 0.0,
        "rel_rmse": 0.0,
    }


def make_raw_entry(values: torch.Tensor) -> Dict[str, object]:
    return {
        "method": "bf16_raw",
        "shape": list(values.shape),
        "dtype": "bfloat16",
        "data": values.to(torch.bfloat16).contiguous(),
    }


@dataclass
class BlockShape:
    """Qwen3-style decoder block.  Defaults: the 2560/9728, 32q/8kv, head 128 block."""
    hidden: int = 2560
    intermediate: int = 9728
    n_heads: int = 32
    n_kv_heads: int = 8
    head_dim: int = 128

    def projections(self) -> List[Tuple[str, int, int]]:
        h, i = self.hidden, self.intermediate
        q = self.n_heads * self.head_dim
        kv = self.n_kv_heads * self.head_dim
        return [
            ("self_attn.q_proj.weight", q, h),
            ("self_attn.k_proj.weight", kv, h),
            ("self_attn.v_proj.weight", kv, h),
            ("self_attn.o_proj.weight", h, q),
            ("mlp.gate_proj.weight", i, h),
            ("mlp.up_proj.weight", i, h),
            ("mlp.down_proj.weight", h, i),
        ]

    def weights_per_block(self) -> int:
        return sum(o * i for _, o, i in self.projections())


# codebook family per projection, as tensor_family() names them
# (compress_full_model.py:256-267) in the default "family" share mode.
FAMILY_OF = {
    "self_attn.q_proj.weight": "attn_q_proj",
    "self_attn.k_proj.weight": "attn_k_proj",
    "self_attn.v_proj.weight": "attn_v_proj",
    "self_attn.o_proj.weight": "attn_o_proj",
    "mlp.gate_proj.weight": "mlp_gate_proj",
    "mlp.up_proj.weight": "mlp_up_proj",
    "mlp.down_proj.weight": "mlp_down_proj",
}


def make_family_codebooks(gen: torch.Generator, stages: int = 4, ncodes: int = 256,
                          d: int = 8) -> Dict[str, torch.Tensor]:
    return {fam: make_codebook(stages, ncodes, d, gen) for fam in FAMILY_OF.values()}


def make_block_entries(shape: BlockShape, layer_idx: int, gen: torch.Generator, *,
                       stages: int = 4, ncodes: int = 256, d: int = 8,
                       group_size: Optional[int] = None,
                       prefix: str = "model.") -> Dict[str, Dict[str, object]]:
    """All entries of one decoder layer: 7 RVQ projections and 4 bf16 norms."""
    entries: Dict[str, Dict[str, object]] = {}
    base = f"{prefix}layers.{layer_idx}."
    for name, o, i in shape.projections():
        entries[base + name] = make_rvq_entry(
            o, i, gen, stages=stages, ncodes=ncodes, d=d, group_size=group_size,
            codebook_id=FAMILY_OF[name])
    for norm, n in (("input_layernorm.weight", shape.hidden),
                    ("post_attention_layernorm.weight", shape.hidden),
                    ("self_attn.q_norm.weight", shape.head_dim),
                    ("self_attn.k_norm.weight", shape.head_dim)):
        w = 1.0 + 0.02 * torch.randn(n, generator=gen)
        entries[base + norm] = make_raw_entry(w)
    return entries


def make_config0_entry(seed: int = 0) -> Tuple[Dict[str, object], torch.Tensor]:
    """Single [9728, 2560] matrix: K=4, 256 codes, d=8, per-row fp16 scales."""
    gen = torch.Generator().manual_seed(seed)
    cb = make_codebook(4, 256, 8, gen)
    entry = make_rvq_entry(9728, 2560, gen, codebook_id="mlp_gate_proj")
    return entry, cb


def make_block_artifact(seed: int = 0, shape: Optional[BlockShape] = None,
                        layer_idx: int = 0) -> Dict[str, object]:
    """One decoder block in artifact form (``format_version`` 1)."""
    shape = shape or BlockShape()
    gen = torch.Generator().manual_seed(seed)
    cbs = make_family_codebooks(gen)
    entries = make_block_entries(shape, layer_idx, gen)
    return {"format_version": 1, "model_type": "qwen3", "shared_codebooks": cbs,
            "entries": entries}


def algorithmic_decode_bytes(entry: Dict[str, object], out_elem_bytes: int = 2,
                             codebook_bytes: int = 0) -> int:
    """Bytes one decode of ``entry`` must move: output write + index, scale and
    tail reads (+ the codebook when given)."""
    numel = 1
    for s in entry["shape"]:
        numel *= int(s)
    idx = entry["indices"]
    return (numel * out_elem_bytes + idx.numel() * idx.element_size()
            + entry["scales"].numel() * entry["scales"].element_size()
            + entry["tail"].numel() * entry["tail"].element_size() + codebook_bytes)


def qwen3_config(shape: BlockShape, n_layers: int, vocab: int, *, rope_theta: float = 1e6,
                 max_positions: int = 4096, rms_eps: float = 1e-6):
    """A Qwen3 config of the given block shape with tied embeddings."""
    from transformers import Qwen3Config
    cfg = Qwen3Config(
        vocab_size=vocab, hidden_size=shape.hidden, intermediate_size=shape.intermediate,
        num_hidden_layers=n_layers, num_attention_heads=shape.n_heads,
        num_key_value_heads=shape.n_kv_heads, head_dim=shape.head_dim,
        max_position_embeddings=max_positions, rms_norm_eps=rms_eps,
        tie_word_embeddings=True, torch_dtype="bfloat16")
    try:
        cfg.rope_theta = rope_theta
        if getattr(cfg, "rope_parameters", None) is not None:
            cfg.rope_parameters["rope_theta"] = rope_theta
    except Exception:
        pass
    cfg._attn_implementation = "eager"
    return cfg


def make_model_artifact(shape: BlockShape, n_layers: int, vocab: int, seed: int = 0, *,
                        stages: int = 4, ncodes: int = 256, group_size: Optional[int] = None,
                        embed_std: float = 0.02) -> Dict[str, object]:
    """A whole random-init model in artifact form: bf16_raw tied embeddings,
    per-layer RVQ projections and bf16 norms, final norm; one codebook per
    projection family (the compressor's default "family" share mode)."""
    gen = torch.Generator().manual_seed(seed)
    cbs = make_family_codebooks(gen, stages=stages, ncodes=ncodes)
    entries: Dict[str, Dict[str, object]] = {}
    embed = torch.randn(vocab, shape.hidden, generator=gen) * embed_std
    entries["model.embed_tokens.weight"] = make_raw_entry(embed)
    for l in range(n_layers):
        entries.update(make_block_entries(shape, l, gen, stages=stages, ncodes=ncodes,
                                          group_size=group_size))
    entries["model.norm.weight"] = make_raw_entry(1.0 + 0.02 * torch.randn(shape.hidden, generator=gen))
    return {"format_version": 1, "model_type": "qwen3", "shared_codebooks": cbs, "entries": entries}


def make_tp_shard_artifact(shape: BlockShape, n_layers: int, vocab: int, rank: int, tp: int, seed: int = 0,
                           device="cpu", embed_std: float = 0.02) -> Dict[str, object]:
    """One rank's shard of a random-init tensor-parallel model, generated on
    ``device`` without building the full model: q/k/v/gate/up hold this rank's
    output rows, o/down its input columns (per-rank seed), while codebooks,
    norms and the tied embedding are replicated (common seed).  The shards of
    all ranks together are one consistent model."""
    if shape.n_heads % tp or shape.n_kv_heads % tp or shape.intermediate % tp:
        raise ValueError("heads and intermediate must split evenly")
    local = BlockShape(hidden=shape.hidden, intermediate=shape.intermediate // tp,
                       n_heads=shape.n_heads // tp, n_kv_heads=shape.n_kv_heads // tp, head_dim=shape.head_dim)
    dev = torch.device(device)
    common = torch.Generator(device=dev).manual_seed(seed)
    mine = torch.Generator(device=dev).manual_seed(seed * 1009 + 7919 * (rank + 1))
    cpu_common = torch.Generator().manual_seed(seed)
    cbs = make_family_codebooks(cpu_common)
    entries: Dict[str, Dict[str, object]] = {}
    embed = torch.randn(vocab, shape.hidden, generator=common, device=dev) * embed_std
    entries["model.embed_tokens.weight"] = make_raw_entry(embed)
    del embed
    for l in range(n_layers):
        base = f"model.layers.{l}."
        for name, o, i in local.projections():
            nvec = o * i // 8
            e = {
                "method": "rvq_groupwise", "codebook_id": FAMILY_OF[name], "shape": [o, i],
                "dtype": "bfloat16", "group_size": int(i), "d": 8, "trimmed_numel": int(o * i),
                "indices": torch.randint(0, 256, (4, nvec), dtype=torch.uint8, generator=mine, device=dev),
                "scales": torch.empty(o, device=dev).uniform_(0.5, 1.5, generator=mine).to(torch.float16),
                "tail": torch.zeros(0, dtype=torch.bfloat16, device=dev), "mse": 0.0, "rel_rmse": 0.0,
            }
            entries[base + name] = e
        for norm, n in (("input_layernorm.weight", shape.hidden), ("post_attention_layernorm.weight", shape.hidden),
                        ("self_attn.q_norm.weight", shape.head_dim), ("self_attn.k_norm.weight", shape.head_dim)):
            entries[base + norm] = make_raw_entry(1.0 + 0.02 * torch.randn(n, generator=common, device=dev))
    entries["model.norm.weight"] = make_raw_entry(1.0 + 0.02 * torch.randn(shape.hidden, generator=common, device=dev))
    return {"format_version": 1, "model_type": "qwen3", "shared_codebooks": cbs, "entries": entries}
