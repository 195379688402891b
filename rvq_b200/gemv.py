"""Fused RVQ dequant-GEMV (batch 1) from Python.

``GemvPlan`` binds up to 4 (entry, codebook, x, y) products -- e.g. the q, k
and v projections of a layer that share x -- to one ``rvq_gemv`` launch
(include/rvq_b200.h), with the C descriptors and the zero-filled workspace
built once and reused.  ``rvq_linear`` is the one-shot form.

The reference has no fused path: it reconstructs each weight into a slot and
calls ``F.linear`` (infer_compressed_layerwise_triton.py:290-292, 296-297).
"""

from __future__ import annotations

import ctypes
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from . import _native
from . import step as _step


class RvqGemvJob(ctypes.Structure):
    _fields_ = [
        ("weight", _native.RvqEntry),
        ("x", ctypes.c_void_p),
        ("y", ctypes.c_void_p),
        ("rows", ctypes.c_int64),
        ("cols", ctypes.c_int64),
        ("x_kind", ctypes.c_int32),
        ("y_kind", ctypes.c_int32),
        ("codes_interleaved", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


_bound = False


def _lib():
    global _bound
    lib = _native.load()
    if not _bound:
        lib.rvq_gemv_workspace_size.restype = ctypes.c_size_t
        lib.rvq_gemv_workspace_size.argtypes = [ctypes.POINTER(RvqGemvJob), ctypes.c_int]
        lib.rvq_gemv.restype = ctypes.c_int
        lib.rvq_gemv.argtypes = [ctypes.POINTER(RvqGemvJob), ctypes.c_int, ctypes.c_void_p,
                                 ctypes.c_size_t, ctypes.c_void_p]
        lib.rvq_interleave_codes.restype = ctypes.c_int
        lib.rvq_interleave_codes.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                             ctypes.c_void_p, ctypes.c_void_p]
        _bound = True
    return lib


def interleave_codes(indices: torch.Tensor) -> torch.Tensor:
    """The [4, nvec] uint8 code planes of an entry as one 32-bit word per
    vector (``[nvec * 4]`` uint8, stage k in byte k): the layout ``rvq_gemv``
    reads with a single load per vector.  Runs on the device."""
    if indices.dtype != torch.uint8 or indices.dim() != 2 or int(indices.shape[0]) != 4:
        raise NotImplementedError("interleaving takes [4, nvec] uint8 code planes")
    indices = indices.contiguous()
    nvec = int(indices.shape[1])
    out = torch.empty(nvec * 4, dtype=torch.uint8, device=indices.device)
    with torch.cuda.device(indices.device):
        rc = _lib().rvq_interleave_codes(ctypes.c_void_p(indices.data_ptr()), nvec, nvec,
                                         ctypes.c_void_p(out.data_ptr()),
                                         ctypes.c_void_p(torch.cuda.current_stream(indices.device).cuda_stream))
    if rc:
        _native.check(rc, "rvq_interleave_codes")
    return out


def gemv_supported(entry: Dict[str, object]) -> bool:
    """Whether ``rvq_gemv`` takes this entry (K=4, 256 codes, uint8 codes,
    no tail, d=8, columns a multiple of 8)."""
    idx = entry["indices"]
    shape = entry["shape"]
    return (entry["method"] in ("rvq_groupwise", "rvq_mlp") and int(entry["d"]) == 8
            and len(shape) == 2 and int(shape[1]) % 8 == 0 and idx.dtype == torch.uint8
            and int(idx.shape[0]) == 4 and entry["tail"].numel() == 0
            and int(entry["trimmed_numel"]) == int(shape[0]) * int(shape[1]))


class GemvPlan:
    """One launch computing ``y_i = W_i x_i`` for every bound product.

    An entry that carries ``"codes_il"`` (from ``interleave_codes``) is read
    in the interleaved layout, else from its artifact code planes."""

    def __init__(self, products: Sequence[Tuple[Dict[str, object], torch.Tensor, torch.Tensor, torch.Tensor]]):
        if not 1 <= len(products) <= 4:
            raise ValueError("a GEMV launch takes 1 to 4 products")
        self._keep: list = []
        jobs: List[RvqGemvJob] = []
        device = None
        for entry, codebook, x, y in products:
            if not gemv_supported(entry):
                raise NotImplementedError(f"rvq_gemv does not take entry of shape {entry['shape']}")
            rows, cols = int(entry["shape"][0]), int(entry["shape"][1])
            if x.numel() != cols or y.numel() != rows or not x.is_contiguous() or not y.is_contiguous():
                raise ValueError("x must have cols elements and y rows elements, both contiguous")
            if codebook.dtype not in (torch.float16, torch.float32):
                codebook = codebook.to(torch.float32)
            if not codebook.is_contiguous() or codebook.data_ptr() % 16:
                codebook = codebook.contiguous().clone()
            scales = entry["scales"] if entry["scales"].is_contiguous() else entry["scales"].contiguous()
            indices = entry["indices"] if entry["indices"].is_contiguous() else entry["indices"].contiguous()
            codes_il = entry.get("codes_il")
            self._keep.append((codebook, scales, indices, x, y, codes_il))
            w = _native.make_entry(indices, codebook, scales, None, y.view(-1), d=8,
                                   group_size=int(entry["group_size"]),
                                   trimmed=int(entry["trimmed_numel"]))
            if codes_il is not None:
                if codes_il.numel() != indices.numel() or codes_il.dtype != torch.uint8:
                    raise ValueError("codes_il does not match the entry's code planes")
                w.indices = codes_il.data_ptr()
            jobs.append(RvqGemvJob(w, x.data_ptr(), y.data_ptr(), rows, cols,
                                   _native.kind_of(x), _native.kind_of(y),
                                   1 if codes_il is not None else 0, 0))
            device = y.device
        self.device = device
        self.jobs = (RvqGemvJob * len(jobs))(*jobs)
        self.n = len(jobs)
        lib = _lib()
        with torch.cuda.device(device):
            nbytes = int(lib.rvq_gemv_workspace_size(self.jobs, self.n))
        self.workspace = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
        self.workspace_bytes = nbytes

    def launch(self, stream: Optional[int] = None) -> None:
        if stream is None:
            stream = torch.cuda.current_stream(self.device).cuda_stream
        rc = _lib().rvq_gemv(self.jobs, self.n, ctypes.c_void_p(self.workspace.data_ptr()),
                             self.workspace_bytes, ctypes.c_void_p(stream))
        if rc:
            _native.check(rc, "rvq_gemv")


def rvq_linear(x: torch.Tensor, entry: Dict[str, object], codebook: torch.Tensor,
               out: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """``F.linear(x, W)`` for one token (x of ``cols`` elements) with W the
    RVQ entry, without materialising W."""
    rows = int(entry["shape"][0])
    if out is None:
        out = torch.empty(rows, dtype=out_dtype or x.dtype, device=x.device)
    GemvPlan([(entry, codebook, x.reshape(-1).contiguous(), out)]).launch()
    return out


# ---------------------------------------------------------------------------
# rvq_gemv_tiles: per-tile partial sums, reduced by the consumer
# ---------------------------------------------------------------------------

class RvqGemvTileJob(ctypes.Structure):
    _fields_ = [
        ("weight", _native.RvqEntry),
        ("x", _step.RvqVec),
        ("gate", _step.RvqVec),
        ("partials", ctypes.c_void_p),
        ("rows", ctypes.c_int64),
        ("cols", ctypes.c_int64),
    ]


_tiles_bound = False


def _tiles_lib():
    global _tiles_bound
    lib = _native.load()
    if not _tiles_bound:
        for name in ("rvq_gemv_tiles", "rvq_gemv_tiles_exact"):
            fn = getattr(lib, name)
            fn.restype = ctypes.c_int
            fn.argtypes = [ctypes.POINTER(RvqGemvTileJob), ctypes.c_int, ctypes.c_void_p]
        lib.rvq_gemv_tiles_count.restype = ctypes.c_int64
        lib.rvq_gemv_tiles_count.argtypes = [ctypes.c_int64]
        lib.rvq_tile_codes_bytes.restype = ctypes.c_int64
        lib.rvq_tile_codes_bytes.argtypes = [ctypes.c_int64, ctypes.c_int64]
        lib.rvq_tile_codes.restype = ctypes.c_int
        lib.rvq_tile_codes.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                       ctypes.c_void_p, ctypes.c_void_p]
        lib.rvq_take_wait_timeout.restype = ctypes.c_int
        lib.rvq_take_wait_timeout.argtypes = []
        _tiles_bound = True
    return lib


def take_wait_timeout() -> bool:
    """True if an ``rvq_gemv_tiles`` wait for its bulk code copies gave up
    since the last call (the result of that launch is then invalid).  Reads
    and clears the library's sticky flag; synchronises the current device."""
    v = _tiles_lib().rvq_take_wait_timeout()
    if v < 0:
        _native.check(-v, "rvq_take_wait_timeout")
    return bool(v)


def tiles_count(cols: int) -> int:
    """Rows of the partials ``rvq_gemv_tiles`` writes for ``cols`` columns."""
    return int(_tiles_lib().rvq_gemv_tiles_count(cols))


def tile_codes(indices: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
    """The [4, nvec] uint8 code planes of a rows x cols entry in the
    tile-major layout ``rvq_gemv_tiles`` streams: ``[tiles, rows, 32]`` 32-bit
    words (stage k in byte k, zero past the last group), returned as a flat
    uint8 tensor.  Runs on the device."""
    if indices.dtype != torch.uint8 or indices.dim() != 2 or int(indices.shape[0]) != 4:
        raise NotImplementedError("tiling takes [4, nvec] uint8 code planes")
    indices = indices.contiguous()
    if int(indices.shape[1]) != rows * (cols // 8) or cols % 8:
        raise ValueError("code planes do not match the weight's shape")
    nbytes = int(_tiles_lib().rvq_tile_codes_bytes(rows, cols))
    out = torch.empty(nbytes, dtype=torch.uint8, device=indices.device)
    with torch.cuda.device(indices.device):
        rc = _tiles_lib().rvq_tile_codes(ctypes.c_void_p(indices.data_ptr()), int(indices.shape[1]), rows, cols,
                                         ctypes.c_void_p(out.data_ptr()),
                                         ctypes.c_void_p(torch.cuda.current_stream(indices.device).cuda_stream))
    if rc:
        _native.check(rc, "rvq_tile_codes")
    return out


class GemvTilesPlan:
    """One ``rvq_gemv_tiles`` launch over up to 4 products.

    ``products``: ``(entry, codebook, x, partials)`` or ``(entry, codebook, x,
    partials, gate)`` tuples.  ``entry["codes_tiled"]`` (from ``tile_codes``)
    is required.  ``x`` / ``gate`` are bf16 vectors or fp32 partials
    ``[ntiles, cols]``; ``partials`` is fp32 ``[tiles_count(cols), rows]``.
    With ``gate`` the operand is ``bf16(bf16(silu(gate)) * x)``.

    ``exact``: ``rvq_gemv_tiles_exact`` -- the weights are the bit-exact bf16
    values of the decoded slot and the products those of ``F.linear`` on it
    (only the fp32 summation order differs); otherwise the lookup-table GEMV,
    whose weights are never rounded to bf16.
    """

    def __init__(self, products, exact: bool = False):
        self.exact = bool(exact)
        self._entry = "rvq_gemv_tiles_exact" if self.exact else "rvq_gemv_tiles"
        if not 1 <= len(products) <= 4:
            raise ValueError("a GEMV launch takes 1 to 4 products")
        self._keep: list = []
        jobs = []
        for prod in products:
            entry, codebook, x, part = prod[:4]
            gate = prod[4] if len(prod) > 4 else None
            if not gemv_supported(entry) or entry.get("codes_tiled") is None:
                raise NotImplementedError("rvq_gemv_tiles needs a K=4 uint8 entry with codes_tiled")
            rows, cols = int(entry["shape"][0]), int(entry["shape"][1])
            nt = tiles_count(cols)
            if part.dtype != torch.float32 or tuple(part.shape) != (nt, rows) or not part.is_contiguous():
                raise ValueError(f"partials must be fp32 [{nt}, {rows}]")
            if codebook.dtype not in (torch.float16, torch.float32):
                codebook = codebook.to(torch.float32)
            if not codebook.is_contiguous() or codebook.data_ptr() % 16:
                codebook = codebook.contiguous().clone()
            scales = entry["scales"].contiguous()
            codes = entry["codes_tiled"]
            xv = _step.vec(x, x.shape[0] if (x.dtype == torch.float32 and x.dim() == 2) else 1)
            gv = _step.vec(gate, gate.shape[0] if (gate is not None and gate.dtype == torch.float32
                                                    and gate.dim() == 2) else 1)
            if xv.n != cols or (gate is not None and gv.n != cols):
                raise ValueError("operand length must equal the weight's columns")
            w = _native.make_entry(entry["indices"], codebook, scales, None, part.view(-1), d=8,
                                   group_size=int(entry["group_size"]), trimmed=int(entry["trimmed_numel"]))
            w.indices = codes.data_ptr()
            self._keep.append((codebook, scales, codes, x, gate, part))
            jobs.append(RvqGemvTileJob(w, xv, gv, part.data_ptr(), rows, cols))
            self.device = part.device
        self.jobs = (RvqGemvTileJob * len(jobs))(*jobs)
        self.n = len(jobs)

    def launch(self, stream: Optional[int] = None) -> None:
        if stream is None:
            stream = torch.cuda.current_stream(self.device).cuda_stream
        rc = getattr(_tiles_lib(), self._entry)(self.jobs, self.n, ctypes.c_void_p(stream))
        if rc:
            _native.check(rc, self._entry)
