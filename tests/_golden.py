"""Loader for the golden vectors in tests/golden (made by make_golden.py)."""

from __future__ import annotations

import glob
import json
import os
from dataclasses import dataclass
from typing import Dict, List

import numpy as np

from oracle.rvq_oracle import (OUT_BF16, OUT_F16, OUT_F32, RVQEntryNP, bf16_bits_to_f32,
                               f16_bits_to_f32)

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
KIND_KEYS = {OUT_F16: "f16", OUT_BF16: "bf16", OUT_F32: "f32"}


@dataclass
class GoldenCase:
    name: str
    meta: dict
    indices: np.ndarray
    codebook_bits: np.ndarray      # uint16 (fp16) or uint32 (fp32) bit patterns
    codebook_is_f16: bool
    scales_f16: np.ndarray         # uint16 bits
    tail_bf16: np.ndarray          # uint16 bits
    expected: Dict[int, np.ndarray]

    @property
    def codebook_f32(self) -> np.ndarray:
        if self.codebook_is_f16:
            return f16_bits_to_f32(self.codebook_bits)
        return self.codebook_bits.view(np.float32)

    def entry_np(self) -> RVQEntryNP:
        shape = self.meta["shape"]
        return RVQEntryNP(
            indices=self.indices, codebook=self.codebook_f32,
            scales=f16_bits_to_f32(self.scales_f16), tail=bf16_bits_to_f32(self.tail_bf16),
            d=int(self.meta["d"]), group_size=int(self.meta["group_size"]),
            trimmed_numel=int(self.meta["trimmed_numel"]), numel=int(np.prod(shape)))

    def entry_torch(self, device="cpu"):
        """The artifact-format entry dict (compress_full_model.py:375-388)."""
        import torch
        return {
            "method": self.meta["method"], "codebook_id": "fixture",
            "shape": list(self.meta["shape"]), "dtype": "bfloat16",
            "group_size": int(self.meta["group_size"]), "d": int(self.meta["d"]),
            "trimmed_numel": int(self.meta["trimmed_numel"]),
            "scales": torch.from_numpy(self.scales_f16.astype(np.int16)).view(torch.float16).to(device),
            "indices": torch.from_numpy(self.indices.copy()).to(device),
            "tail": torch.from_numpy(self.tail_bf16.astype(np.int16)).view(torch.bfloat16).to(device),
            "mse": 0.0, "rel_rmse": 0.0,
        }

    def codebook_torch(self, device="cpu", dtype=None):
        import torch
        if self.codebook_is_f16:
            cb = torch.from_numpy(self.codebook_bits.astype(np.int16)).view(torch.float16)
        else:
            cb = torch.from_numpy(self.codebook_bits.astype(np.int32)).view(torch.float32)
        cb = cb.to(device)
        return cb if dtype is None else cb.to(dtype)


def case_names() -> List[str]:
    """RVQ decode fixtures (others: engine_*, int8_*, encoder_* and proj_* files)."""
    return sorted(os.path.splitext(os.path.basename(p))[0]
                  for p in glob.glob(os.path.join(GOLDEN_DIR, "*.npz"))
                  if not os.path.basename(p).startswith(("engine_", "int8_", "encoder_", "proj_")))


def int8_case_names() -> List[str]:
    """int8_groupwise fixtures (made by make_golden_int8.py)."""
    return sorted(os.path.splitext(os.path.basename(p))[0]
                  for p in glob.glob(os.path.join(GOLDEN_DIR, "int8_*.npz")))


@dataclass
class Int8Case:
    name: str
    meta: dict
    q: np.ndarray                  # int8 [trimmed]
    scales_f16: np.ndarray         # uint16 bits, one per group
    tail_bf16: np.ndarray          # uint16 bits
    expected: Dict[int, np.ndarray]

    def entry_torch(self, device="cpu"):
        """The artifact-format entry dict (compress_full_model.py:414-425)."""
        import torch
        gs = int(self.meta["group_size"])
        return {
            "method": "int8_groupwise", "shape": list(self.meta["shape"]), "dtype": "bfloat16",
            "group_size": gs, "trimmed_numel": int(self.meta["trimmed_numel"]),
            "q": torch.from_numpy(self.q.copy()).view(-1, gs).to(device),
            "scales": torch.from_numpy(self.scales_f16.astype(np.int16)).view(torch.float16).to(device),
            "tail": torch.from_numpy(self.tail_bf16.astype(np.int16)).view(torch.bfloat16).to(device),
            "mse": 0.0, "rel_rmse": 0.0,
        }


def load_int8_case(name: str) -> Int8Case:
    z = np.load(os.path.join(GOLDEN_DIR, f"{name}.npz"))
    meta = json.loads(bytes(z["meta_json"]).decode())
    expected = {kind: z[f"expected_{key}"] for kind, key in KIND_KEYS.items()}
    return Int8Case(name=name, meta=meta, q=z["q"], scales_f16=z["scales_f16"], tail_bf16=z["tail_bf16"],
                    expected=expected)


def load_case(name: str) -> GoldenCase:
    z = np.load(os.path.join(GOLDEN_DIR, f"{name}.npz"))
    meta = json.loads(bytes(z["meta_json"]).decode())
    is_f16 = "codebook_f16" in z.files
    cb = z["codebook_f16"] if is_f16 else z["codebook_f32"]
    expected = {kind: z[f"expected_{key}"] for kind, key in KIND_KEYS.items()}
    return GoldenCase(name=name, meta=meta, indices=z["indices"], codebook_bits=cb,
                      codebook_is_f16=is_f16, scales_f16=z["scales_f16"],
                      tail_bf16=z["tail_bf16"], expected=expected)


def load_checksums() -> dict:
    with open(os.path.join(GOLDEN_DIR, "checksums.json")) as f:
        return json.load(f)


def bits_equal(got: np.ndarray, want: np.ndarray, out_kind: int) -> bool:
    """Bitwise equality, except that any NaN equals any NaN (payloads differ
    between conversion routines and carry no value)."""
    got = np.asarray(got).reshape(-1)
    want = np.asarray(want).reshape(-1)
    if got.shape != want.shape:
        return False
    if out_kind == OUT_F32:
        gv, wv = got.view(np.float32), want.view(np.float32)
    elif out_kind == OUT_F16:
        gv, wv = f16_bits_to_f32(got), f16_bits_to_f32(want)
    else:
        gv, wv = bf16_bits_to_f32(got), bf16_bits_to_f32(want)
    nan = np.isnan(gv) & np.isnan(wv)
    return bool(np.all((got == want) | nan))


def load_projection() -> dict:
    """The reference-encoded [1024, 2560] entry at group size 128
    (make_golden_projection.py): planes, fp16 scales and codebooks, and the
    sha256 of the reference's decode per output kind."""
    z = np.load(os.path.join(GOLDEN_DIR, "proj_k_g128.npz"))
    out = {k: z[k] for k in ("indices", "scales_f16", "codebook_f16")}
    out["sha256"] = {kind: bytes(z[f"sha256_{key}"]).decode() for kind, key in KIND_KEYS.items()}
    return out
