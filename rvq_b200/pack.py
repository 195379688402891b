"""Artifact packs: the compressor's artifact as one flat file, loaded natively.

The reference stores the compressed model with ``torch.save`` (a pickle,
compress_full_model.py:624-631) and its engines ``torch.load`` it and move
every tensor to the GPU one by one (infer_compressed_layerwise_triton.py:
421-432).  A pack holds the same dict:

    bytes 0..7      b"RVQPACK1"
    bytes 8..15     little-endian u64: length L of the JSON header
    bytes 16..23    little-endian u64: length D of the data region
    bytes 24..24+L  UTF-8 JSON: every non-tensor field as is; a tensor is
                    {"__tensor__": [offset, nbytes], "dtype": ..., "shape": [...]}
    from DATA       the tensors' bytes, each at a 4096-byte aligned offset
                    (relative to DATA, the first 4096-byte boundary after the header)

``read_pack`` parses the header in Python and loads the whole data region
into ONE device buffer with ``rvq_pack_load`` (C++: pread into a ring of
pinned buffers on a reader thread, overlapped with the host-to-device
copies); every tensor of the returned dict is a view into that buffer.
"""

from __future__ import annotations

import ctypes
import json
import os
import struct
from typing import Dict, Tuple

import torch

from . import _native

MAGIC = b"RVQPACK1"
ALIGN = 4096

_DTYPES = {
    "uint8": torch.uint8, "int8": torch.int8, "int16": torch.int16, "int32": torch.int32, "int64": torch.int64,
    "float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32,
}
_NAMES = {v: k for k, v in _DTYPES.items()}


def _align(n: int) -> int:
    return -(-n // ALIGN) * ALIGN


def write_pack(artifact: Dict[str, object], path: str) -> int:
    """Write ``artifact`` (the compressor's dict of codebooks and entries) as a
    pack.  Returns the file size."""
    blobs = []
    offset = 0

    def enc(v):
        nonlocal offset
        if torch.is_tensor(v):
            t = v.detach().contiguous().cpu()
            if t.dtype not in _NAMES:
                raise NotImplementedError(f"pack cannot hold {t.dtype}")
            nbytes = t.numel() * t.element_size()
            desc = {"__tensor__": [offset, nbytes], "dtype": _NAMES[t.dtype], "shape": list(t.shape)}
            blobs.append((offset, t))
            offset = _align(offset + nbytes)
            return desc
        if isinstance(v, dict):
            return {str(k): enc(x) for k, x in v.items()}
        if isinstance(v, (list, tuple)):
            return [enc(x) for x in v]
        return v

    header = json.dumps(enc(artifact)).encode()
    data_start = _align(24 + len(header))
    with open(path, "wb") as f:
        f.write(MAGIC)
        f.write(struct.pack("<QQ", len(header), offset))
        f.write(header)
        for off, t in blobs:
            f.seek(data_start + off)
            f.write(t.view(torch.uint8).reshape(-1).numpy().tobytes() if t.numel() else b"")
        end = data_start + offset
        f.truncate(end)
    return end


def read_header(path: str) -> Tuple[dict, int, int]:
    """(header dict, byte offset of the data region, its length)."""
    with open(path, "rb") as f:
        if f.read(8) != MAGIC:
            raise ValueError(f"{path} is not an artifact pack")
        n, data_len = struct.unpack("<QQ", f.read(16))
        header = json.loads(f.read(n).decode())
    data_start = _align(24 + n)
    if os.path.getsize(path) < data_start + data_len:
        raise ValueError(f"{path} is truncated: its data region is shorter than the header says")
    return header, data_start, data_len


def read_pack(path: str, device) -> Dict[str, object]:
    """The artifact dict with every tensor on ``device``, views into one buffer."""
    header, data_start, nbytes = read_header(path)
    device = torch.device(device)
    buf = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=device)
    lib = _native.load()
    lib.rvq_pack_load.restype = ctypes.c_int
    lib.rvq_pack_load.argtypes = [ctypes.c_char_p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_void_p,
                                  ctypes.c_void_p]
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device).cuda_stream
        _native.check(lib.rvq_pack_load(os.fsencode(path), data_start, nbytes, ctypes.c_void_p(buf.data_ptr()),
                                        ctypes.c_void_p(stream)), "rvq_pack_load")

    def dec(v):
        if isinstance(v, dict):
            if "__tensor__" in v:
                off, n = v["__tensor__"]
                dt = _DTYPES[v["dtype"]]
                return buf[off:off + n].view(dt).view(v["shape"])
            return {k: dec(x) for k, x in v.items()}
        if isinstance(v, list):
            return [dec(x) for x in v]
        return v

    return dec(header)
