"""Decode dispatch of the layerwise engine, B200 edition.

Mirrors the reference's engine-level entry points so they stay drop-ins:

* ``decode_into(entry, codebooks, out)``  -- infer_compressed_layerwise_triton.py:161-176
* ``decode_to_tensor(entry, codebooks, device, runtime_dtype)`` -- same file, 179-188

(``int8_groupwise`` entries, which the reference's Triton engine rejects,
decode here as in the single-slot engine),

and adds ``LayerDecodePlan``: all entries of one decoder layer (7 RVQ
projections + 4 bf16 norm copies for Qwen3) decoded by ONE kernel launch,
with the C descriptors built once and reused every time the layer is
decoded.  It replaces the per-key loop of ``prefetch_layer``
(infer_compressed_layerwise_triton.py:246-266).
"""

from __future__ import annotations

import ctypes
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from . import _native
from .triton_decode_kernels import decode_rvq_triton_into, prepare_entry, rvq_triton_supported

RVQ_METHODS = ("rvq_groupwise", "rvq_mlp")


def prepare_int8_entry(entry: Dict[str, object], out: torch.Tensor):
    """Validate an int8_groupwise entry (compress_full_model.py:414-425) for
    ``out`` and return (C struct, tensors to keep alive)."""
    if not out.is_cuda or not out.is_contiguous():
        raise ValueError("Output tensor must be a contiguous CUDA tensor.")
    q, scales, tail = entry["q"], entry["scales"], entry["tail"]
    for name, t in (("q", q), ("scales", scales), ("tail", tail)):
        if t.numel() and not t.is_cuda:
            raise ValueError(f"Entry tensor {name} must be on CUDA.")
    if q.dtype != torch.int8:
        raise NotImplementedError(f"int8_groupwise codes must be int8, got {q.dtype}")
    trimmed, group_size = int(entry["trimmed_numel"]), int(entry["group_size"])
    if q.numel() != trimmed or out.numel() < trimmed + tail.numel():
        raise ValueError("int8 entry does not match the output tensor")
    q = q.contiguous()
    if scales.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        scales = scales.to(torch.float32)
    scales = scales.contiguous()
    tail = tail.contiguous()
    st = _native.make_int8_entry(q, scales, tail, out.view(-1), group_size=group_size, trimmed=trimmed)
    return st, (q, scales, tail)


def decode_int8_into(entry: Dict[str, object], out: torch.Tensor) -> torch.Tensor:
    """One int8_groupwise entry into ``out`` on the current stream: the
    single-slot engine's ``_decode_int8_into``
    (infer_compressed_layerwise_single_slot.py:110-120) on the GPU."""
    st, keep = prepare_int8_entry(entry, out)
    with torch.cuda.device(out.device):
        _native.check(_native.load().rvq_decode_int8(ctypes.byref(st), ctypes.c_void_p(
            torch.cuda.current_stream(out.device).cuda_stream)), "rvq_decode_int8")
    del keep
    return out


def decode_into(entry: Dict[str, object], codebooks: Dict[str, torch.Tensor], out: torch.Tensor):
    """Reference: infer_compressed_layerwise_triton.py:161-176.  The reference
    engine raises for ``int8_groupwise`` entries; this one decodes them as the
    single-slot engine does (infer_compressed_layerwise_single_slot.py:155-157)."""
    method = entry["method"]
    if method == "bf16_raw":
        flat_data = entry["data"].view(torch.int16)
        out.view(torch.int16).copy_(flat_data, non_blocking=True)
    elif method == "int8_groupwise":
        decode_int8_into(entry, out)
    elif method in RVQ_METHODS:
        codebook = codebooks[entry["codebook_id"]]
        if not rvq_triton_supported(entry, out):
            raise ValueError(f"Triton kernel does not support entry shape {entry['shape']}")
        decode_rvq_triton_into(entry, codebook, out)
    else:
        raise ValueError(f"Unsupported decode method: {method}")


def decode_to_tensor(entry: Dict[str, object], codebooks: Dict[str, torch.Tensor],
                     device: torch.device, runtime_dtype: torch.dtype) -> torch.Tensor:
    """Reference: infer_compressed_layerwise_triton.py:179-188."""
    shape = tuple(entry["shape"])
    out = torch.empty(shape, dtype=runtime_dtype, device=device)
    decode_into(entry, codebooks, out)
    return out


class LayerDecodePlan:
    """Everything one layer-slot fill needs, resolved once.

    ``items``: ``(key, entry)`` pairs of one layer; ``outs[key]``: the slot
    tensor each entry decodes into; ``max_ctas``: CTA budget of the launch (0:
    one CTA per SM; fewer leaves SMs to the kernels of the layer being computed);
    ``quad_codes``: repack eligible entries' codes once into the quad layout
    the slot kernel streams with one 16-byte load per 4 vectors (the entries'
    own planes are left as they are).  ``launch(stream)`` queues the whole
    layer as ceil(jobs / 32) launches (one for a Qwen3 layer: 11 jobs).
    The tensors referenced by the plan must outlive it.
    """

    def __init__(self, items: Sequence[Tuple[str, Dict[str, object]]],
                 codebooks: Dict[str, torch.Tensor], outs: Dict[str, torch.Tensor], max_ctas: int = 0,
                 quad_codes: bool = True):
        self.keys: List[str] = []
        fp16_codebooks: Dict[int, Optional[torch.Tensor]] = {}
        entries: List[_native.RvqEntry] = []
        int8s: List[_native.RvqInt8Entry] = []
        copies: List[Tuple[int, int, int]] = []
        self._keep: list = []
        self.algorithmic_bytes = 0
        for key, entry in items:
            out = outs[key]
            method = entry["method"]
            if method == "bf16_raw":
                data = entry["data"]
                if not data.is_cuda or not out.is_cuda:
                    raise ValueError("bf16_raw copy needs CUDA source and slot tensors")
                if data.element_size() != 2 or out.element_size() != 2:
                    raise ValueError("bf16_raw copy is a 16-bit view copy")
                if data.numel() != out.numel() or not out.is_contiguous():
                    raise ValueError(f"slot for {key} does not match its bf16_raw entry")
                data = data.contiguous()
                self._keep.append(data)
                nbytes = data.numel() * 2
                copies.append((data.data_ptr(), out.data_ptr(), nbytes))
                self.algorithmic_bytes += 2 * nbytes
            elif method == "int8_groupwise":
                st, keep = prepare_int8_entry(entry, out)
                self._keep.append(keep)
                int8s.append(st)
                self.algorithmic_bytes += (out.numel() * out.element_size() + entry["q"].numel()
                                           + entry["scales"].numel() * entry["scales"].element_size()
                                           + entry["tail"].numel() * entry["tail"].element_size())
            elif method in RVQ_METHODS:
                cb = codebooks[entry["codebook_id"]]
                if not rvq_triton_supported(entry, out):
                    raise ValueError(f"Triton kernel does not support entry shape {entry['shape']}")
                st, keep = prepare_entry(entry, cb, out)
                self._keep.append(keep)
                if quad_codes:
                    self._to_quad(st, entry, cb, out, fp16_codebooks)
                entries.append(st)
                idx = entry["indices"]
                self.algorithmic_bytes += (out.numel() * out.element_size()
                                           + idx.numel() * idx.element_size()
                                           + entry["scales"].numel() * entry["scales"].element_size()
                                           + entry["tail"].numel() * entry["tail"].element_size())
            else:
                raise ValueError(f"Unsupported decode method: {method}")
            self.keys.append(key)
        self.batches = []
        jobs = [("e", e) for e in entries] + [("i", e) for e in int8s] + [("c", c) for c in copies]
        for i in range(0, len(jobs), _native.RVQ_MAX_LAYER_JOBS):
            chunk = jobs[i:i + _native.RVQ_MAX_LAYER_JOBS]
            es = [j for t, j in chunk if t == "e"]
            qs = [j for t, j in chunk if t == "i"]
            cs = [j for t, j in chunk if t == "c"]
            earr = (_native.RvqEntry * max(len(es), 1))(*es)
            qarr = (_native.RvqInt8Entry * max(len(qs), 1))(*qs)
            carr = (_native.RvqCopy * max(len(cs), 1))(*[_native.RvqCopy(*c) for c in cs])
            self.batches.append((earr, len(es), qarr, len(qs), carr, len(cs)))
        self._lib = _native.load()
        self.max_ctas = int(max_ctas)

    def _to_quad(self, st: _native.RvqEntry, entry, codebook: torch.Tensor, out: torch.Tensor,
                 fp16_codebooks: Dict[int, Optional[torch.Tensor]]) -> None:
        """Point ``st`` at a one-time repack of its codes into the quad layout
        (rvq_quad_codes) and at an fp16 copy of its codebook, when the entry
        is one the slot kernel decodes: 4 stages of 256 uint8 codes, every
        codebook value an exact fp16 number (checked once per codebook), a
        bf16 slot, fp16 scales, whole vectors, a multiple of 4 vectors per
        scale.  Otherwise ``st`` keeps the artifact's planes."""
        idx = entry["indices"]
        nvec = int(idx.shape[1]) if idx.dim() == 2 else 0
        if not (idx.dtype == torch.uint8 and idx.dim() == 2 and int(idx.shape[0]) == 4 and nvec > 0
                and int(codebook.shape[1]) == 256 and out.dtype == torch.bfloat16
                and entry["scales"].dtype == torch.float16 and int(entry["trimmed_numel"]) == nvec * 8
                and (int(entry["group_size"]) // 8) % 4 == 0 and out.data_ptr() % 32 == 0):
            return
        key = id(codebook)
        if key not in fp16_codebooks:
            h = codebook.to(torch.float16).contiguous()
            fp16_codebooks[key] = h if torch.equal(h.to(codebook.dtype), codebook) else None
        h = fp16_codebooks[key]
        if h is None:
            return
        lib = _native.load()
        lib.rvq_quad_codes_bytes.restype = ctypes.c_int64
        lib.rvq_quad_codes_bytes.argtypes = [ctypes.c_int64]
        lib.rvq_quad_codes.restype = ctypes.c_int
        lib.rvq_quad_codes.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
                                       ctypes.c_void_p]
        planes = idx.contiguous()
        quads = torch.empty(int(lib.rvq_quad_codes_bytes(nvec)), dtype=torch.uint8, device=idx.device)
        with torch.cuda.device(idx.device):
            _native.check(lib.rvq_quad_codes(ctypes.c_void_p(planes.data_ptr()), nvec, nvec,
                                             ctypes.c_void_p(quads.data_ptr()),
                                             ctypes.c_void_p(torch.cuda.current_stream(idx.device).cuda_stream)),
                          "rvq_quad_codes")
        self._keep.append((quads, h))
        st.indices = quads.data_ptr()
        st.stage_stride = nvec
        st.index_kind = _native.RVQ_U8X4
        st.codebook = h.data_ptr()
        st.codebook_kind = _native.RVQ_F16

    @property
    def launches(self) -> int:
        return len(self.batches)

    def launch(self, stream: Optional[int] = None) -> None:
        if stream is None:
            stream = torch.cuda.current_stream().cuda_stream
        s = ctypes.c_void_p(stream)
        for earr, ne, qarr, nq, carr, nc in self.batches:
            rc = self._lib.rvq_decode_layer_ctas(earr, ne, qarr, nq, carr, nc, self.max_ctas, s)
            if rc:
                _native.check(rc, "rvq_decode_layer_ctas")
