"""Tensor-parallel reduction of the row-parallel projections over NVLink peer
memory (include/rvq_b200.h: ``rvq_tp_push``, ``rvq_p2p_alloc``,
``rvq_ipc_export`` / ``rvq_ipc_import``).

Each rank owns one device block holding, per reduction point (``o`` after
attention, ``down`` after the MLP), an arrival counter, the count of arrivals
it has consumed, and one landing buffer [tp][hidden] fp32.  After a
row-parallel projection the rank launches one push kernel that sums its own
output and stores it into slot [rank] of every rank's landing buffer, then
bumps every rank's counter.  The next RMSNorm (``NormOp`` with ``landing``)
waits for the counter, adds the tp slots in rank order and advances its
consumed count: an all-reduce in two of the step's own launches, with no
collective library call in the decode step.

Why one landing buffer per reduction point suffices (no double buffering):
rank B writes its slot of rank A's ``o`` buffer for layer l+1 only after B's
norm after ``down`` of layer l has seen A's ``down`` push of layer l, and A
launches that push after it has finished reading its ``o`` buffer for layer
l.  The same argument holds for ``down`` with the roles of the two points
exchanged.  Each point has its own counter, so arrivals for one point can
never satisfy a wait at the other: a peer's late ``o`` push of layer l is
never counted toward this rank's ``down`` wait of layer l.

Setup is collective: every rank of the group constructs ``PeerExchange`` at
the same point, and ``close()`` is collective too.
"""

from __future__ import annotations

import ctypes
from typing import Dict, Optional

import torch
import torch.distributed as dist

from . import _native
from .step import RvqVec

RVQ_MAX_TP = 8
_HEADER = 256                  # per point: arrivals (u32) and consumed (u32), padded to 256 B


class RvqTpPushArgs(ctypes.Structure):
    _fields_ = [("src", RvqVec), ("dst", ctypes.c_void_p * RVQ_MAX_TP),
                ("arrivals", ctypes.c_void_p * RVQ_MAX_TP), ("n", ctypes.c_int64),
                ("rank", ctypes.c_int32), ("tp", ctypes.c_int32)]


_bound = False


def _lib():
    global _bound
    lib = _native.load()
    if not _bound:
        vp, i32 = ctypes.c_void_p, ctypes.c_int
        lib.rvq_tp_push_ctas.restype = ctypes.c_uint32
        lib.rvq_tp_push_ctas.argtypes = [ctypes.c_int64]
        lib.rvq_tp_push.restype = i32
        lib.rvq_tp_push.argtypes = [ctypes.POINTER(RvqTpPushArgs), vp]
        lib.rvq_p2p_alloc.restype = i32
        lib.rvq_p2p_alloc.argtypes = [ctypes.c_size_t, ctypes.POINTER(vp)]
        lib.rvq_p2p_free.restype = i32
        lib.rvq_p2p_free.argtypes = [vp]
        lib.rvq_ipc_export.restype = i32
        lib.rvq_ipc_export.argtypes = [vp, ctypes.c_char_p]
        lib.rvq_ipc_import.restype = i32
        lib.rvq_ipc_import.argtypes = [ctypes.c_char_p, ctypes.POINTER(vp)]
        lib.rvq_ipc_close.restype = i32
        lib.rvq_ipc_close.argtypes = [vp]
        lib.rvq_take_tp_timeout.restype = i32
        lib.rvq_take_tp_timeout.argtypes = []
        _bound = True
    return lib


def push_ctas(n: int) -> int:
    """Arrivals one rank's push of an n-vector adds to every counter."""
    return int(_lib().rvq_tp_push_ctas(n))


def take_timeout() -> bool:
    """True if a landing-buffer wait gave up since the last call (synchronises)."""
    v = _lib().rvq_take_tp_timeout()
    if v < 0:
        _native.check(-v, "rvq_take_tp_timeout")
    return bool(v)


class DeviceBlock:
    """Zero-filled ``rvq_p2p_alloc`` memory of this process."""

    def __init__(self, nbytes: int):
        p = ctypes.c_void_p()
        _native.check(_lib().rvq_p2p_alloc(nbytes, ctypes.byref(p)), "rvq_p2p_alloc")
        self.ptr, self.nbytes = int(p.value), nbytes

    def handle(self) -> bytes:
        h = ctypes.create_string_buffer(64)
        _native.check(_lib().rvq_ipc_export(self.ptr, h), "rvq_ipc_export")
        return h.raw

    def free(self) -> None:
        if self.ptr:
            _native.check(_lib().rvq_p2p_free(self.ptr), "rvq_p2p_free")
            self.ptr = 0


def _import(handle: bytes) -> int:
    p = ctypes.c_void_p()
    _native.check(_lib().rvq_ipc_import(handle, ctypes.byref(p)), "rvq_ipc_import")
    return int(p.value)


class PeerExchange:
    """Landing buffers, counters and peer mappings of one tensor-parallel group."""

    POINTS = ("o", "down")

    def __init__(self, group, hidden: int, device: torch.device):
        self.group = group
        self.tp = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if not 1 < self.tp <= RVQ_MAX_TP:
            raise ValueError(f"peer exchange needs 2..{RVQ_MAX_TP} ranks")
        self.hidden = hidden
        self.device = torch.device(device)
        land = -(-self.tp * hidden * 4 // 256) * 256
        self.offsets = {p: _HEADER + i * land for i, p in enumerate(self.POINTS)}
        with torch.cuda.device(self.device):
            self.block = DeviceBlock(_HEADER + len(self.POINTS) * land)
            handles = [None] * self.tp
            dist.all_gather_object(handles, self.block.handle(), group=group)
            self.bases = []
            self._imported = []
            for r, h in enumerate(handles):
                if r == self.rank:
                    self.bases.append(self.block.ptr)
                else:
                    b = _import(h)
                    self._imported.append(b)
                    self.bases.append(b)
        self.arrivals_per_use = self.tp * push_ctas(hidden)

    # local pointers read by the consuming norm kernel
    def landing(self, point: str) -> Dict[str, int]:
        c = self.counters(point)
        return {"add": self.block.ptr + self.offsets[point], "arrivals": self.block.ptr + c,
                "consumed": self.block.ptr + c + 4, "per_use": self.arrivals_per_use, "tp": self.tp}

    def counters(self, point: str) -> int:
        """Byte offset of the point's (arrivals, consumed) pair in a block."""
        return 8 * self.POINTS.index(point)

    def push_args(self, point: str, src: RvqVec) -> RvqTpPushArgs:
        a = RvqTpPushArgs()
        a.src = src
        for r in range(self.tp):
            a.dst[r] = self.bases[r] + self.offsets[point]
            a.arrivals[r] = self.bases[r] + self.counters(point)
        a.n, a.rank, a.tp = self.hidden, self.rank, self.tp
        return a

    def close(self) -> None:
        """Collective: unmap the peers' blocks and free this rank's."""
        if self.block.ptr == 0:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)            # no peer still writes into this block
        with torch.cuda.device(self.device):
            for b in self._imported:
                _native.check(_lib().rvq_ipc_close(b), "rvq_ipc_close")
            self._imported = []
            dist.barrier(group=self.group)        # every peer has unmapped this block
            self.block.free()

    def __del__(self):
        # not collective: unmap the peers, leave this rank's block to process exit
        try:
            if self.block.ptr and self._imported:
                for b in self._imported:
                    _lib().rvq_ipc_close(b)
                self._imported = []
        except Exception:
            pass


class TpPushOp:
    """One ``rvq_tp_push`` launch of this rank's projection output into ``point``."""

    def __init__(self, exchange: PeerExchange, point: str, src: torch.Tensor, src_tiles: int = 1):
        from .step import vec
        if src.numel() != exchange.hidden * src_tiles:
            raise ValueError("the pushed vector must have the exchange's hidden size")
        self._keep = (exchange, src)
        self.args = exchange.push_args(point, vec(src, src_tiles))

    def launch(self) -> None:
        rc = _lib().rvq_tp_push(ctypes.byref(self.args), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        if rc:
            _native.check(rc, "rvq_tp_push")
