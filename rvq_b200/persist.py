"""The persistent batch-1 decode step from Python (``rvq_persist_*``,
include/rvq_b200.h).

One cooperative launch per token runs every layer of a fused-mode
``Qwen3Decoder`` -- norms, the four table GEMVs, attention -- and the final
norm; only the vocabulary head (``F.linear`` on the final-normed hidden state)
stays a separate call.  It replaces the seven launches per layer of the plain
native step (the reference's per-layer module calls in ``_layerwise_logits``,
infer_compressed_layerwise_triton.py:271-292) and is bit-identical to it.
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _native

SYNC_WORDS = 1024        # RVQ_PERSIST_SYNC_WORDS


class RvqPersistLayer(ctypes.Structure):
    _fields_ = [("proj", _native.RvqEntry * 7), ("input_norm", ctypes.c_void_p),
                ("post_norm", ctypes.c_void_p), ("q_norm", ctypes.c_void_p), ("k_norm", ctypes.c_void_p),
                ("k_cache", ctypes.c_void_p), ("v_cache", ctypes.c_void_p)]


class RvqPersistModel(ctypes.Structure):
    _fields_ = [("n_layers", ctypes.c_int32), ("hidden", ctypes.c_int32), ("intermediate", ctypes.c_int32),
                ("n_heads", ctypes.c_int32), ("n_kv", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("max_len", ctypes.c_int32), ("vocab", ctypes.c_int32), ("eps", ctypes.c_float),
                ("scaling", ctypes.c_float), ("valid_bias", ctypes.c_float), ("reserved", ctypes.c_int32),
                ("embed", ctypes.c_void_p), ("final_norm", ctypes.c_void_p), ("cos", ctypes.c_void_p),
                ("sin", ctypes.c_void_p), ("token", ctypes.c_void_p), ("pos", ctypes.c_void_p),
                ("h", ctypes.c_void_p), ("x_final", ctypes.c_void_p), ("attn_out", ctypes.c_void_p),
                ("q_part", ctypes.c_void_p), ("k_part", ctypes.c_void_p), ("v_part", ctypes.c_void_p),
                ("o_part", ctypes.c_void_p), ("gate_part", ctypes.c_void_p), ("up_part", ctypes.c_void_p),
                ("down_part", ctypes.c_void_p), ("sync", ctypes.c_void_p)]


_bound = False


def _lib():
    global _bound
    lib = _native.load()
    if not _bound:
        lib.rvq_persist_plan_bytes.restype = ctypes.c_int64
        lib.rvq_persist_plan_bytes.argtypes = [ctypes.POINTER(RvqPersistModel), ctypes.POINTER(RvqPersistLayer)]
        lib.rvq_persist_plan.restype = ctypes.c_int
        lib.rvq_persist_plan.argtypes = [ctypes.POINTER(RvqPersistModel), ctypes.POINTER(RvqPersistLayer),
                                         ctypes.c_void_p, ctypes.c_int64]
        lib.rvq_persist_plan_for.restype = ctypes.c_int64
        lib.rvq_persist_plan_for.argtypes = [ctypes.POINTER(RvqPersistModel), ctypes.POINTER(RvqPersistLayer),
                                             ctypes.c_int32, ctypes.c_void_p, ctypes.c_int64]
        lib.rvq_persist_step.restype = ctypes.c_int
        lib.rvq_persist_step.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        lib.rvq_persist_take_error.restype = ctypes.c_int
        lib.rvq_persist_take_error.argtypes = []
        _bound = True
    return lib


def _ptr(t: torch.Tensor) -> int:
    return t.data_ptr()


class PersistentStep:
    """The step plan of a fused-mode decoder (native step ops built, one
    GPU).  ``launch()`` enqueues one decode step for the token in
    ``dec._tok`` at ``dec._pos``: ``dec.h`` / ``dec.x_final`` and the KV cache
    are then exactly what the plain native step leaves."""

    def __init__(self, dec):
        if dec.mode != "fused" or dec.tp != 1 or dec.step_impl not in ("native", "persistent"):
            raise NotImplementedError("the persistent step runs a single-GPU decoder in fused mode")
        d, dev = dec.dims, dec.device
        self.device = dev
        self.sync = torch.zeros(SYNC_WORDS, dtype=torch.int32, device=dev)
        m = RvqPersistModel()
        m.n_layers, m.hidden, m.intermediate = d.n_layers, d.hidden, d.intermediate
        m.n_heads, m.n_kv, m.head_dim = d.n_heads, d.n_kv, d.head_dim
        m.max_len, m.vocab = dec.max_len, int(dec.embed.shape[0])
        m.eps, m.scaling, m.valid_bias = d.eps, dec.scaling, 0.0 if dec.causal else 1.0
        m.reserved = 0
        m.embed, m.final_norm = _ptr(dec.embed), _ptr(dec.final_norm)
        m.cos, m.sin = _ptr(dec.cos), _ptr(dec.sin)
        m.token, m.pos = _ptr(dec._tok), _ptr(dec._pos)
        m.h, m.x_final, m.attn_out = _ptr(dec.h), _ptr(dec.x_final), _ptr(dec.attn_out)
        m.q_part, m.k_part, m.v_part = _ptr(dec.q_part), _ptr(dec.k_part), _ptr(dec.v_part)
        m.o_part, m.gate_part, m.up_part = _ptr(dec.o_part), _ptr(dec.gate_part), _ptr(dec.up_part)
        m.down_part, m.sync = _ptr(dec.down_part), _ptr(self.sync)
        layers = (RvqPersistLayer * d.n_layers)()
        for l, (L, ops) in enumerate(zip(dec.layers, dec.step_ops)):
            Y = layers[l]
            weights = [ops["qkv"].jobs[i].weight for i in range(3)] + [ops["o"].jobs[0].weight] + \
                      [ops["gu"].jobs[i].weight for i in range(2)] + [ops["down"].jobs[0].weight]
            for i, w in enumerate(weights):
                Y.proj[i] = w
            Y.input_norm = _ptr(L["input_layernorm.weight"])
            Y.post_norm = _ptr(L["post_attention_layernorm.weight"])
            Y.q_norm = _ptr(L["self_attn.q_norm.weight"])
            Y.k_norm = _ptr(L["self_attn.k_norm.weight"])
            Y.k_cache, Y.v_cache = _ptr(dec.k_cache[l]), _ptr(dec.v_cache[l])
        self._layers = layers               # the decoder owns every buffer the plan points at
        lib = _lib()
        with torch.cuda.device(dev):
            nbytes = lib.rvq_persist_plan_bytes(ctypes.byref(m), layers)
            if nbytes <= 0:                 # the planner's status says why
                probe = torch.zeros(16, dtype=torch.uint8)
                rc = lib.rvq_persist_plan(ctypes.byref(m), layers, ctypes.c_void_p(probe.data_ptr()), 16)
                _native.check(rc or _native.RVQ_ERR_UNAVAILABLE, "rvq_persist_plan_bytes")
            host = torch.zeros(int(nbytes), dtype=torch.uint8)
            rc = lib.rvq_persist_plan(ctypes.byref(m), layers, ctypes.c_void_p(host.data_ptr()), int(nbytes))
            if rc:
                _native.check(rc, "rvq_persist_plan")
        self.plan = host.to(dev)
        self.plan_bytes = int(nbytes)

    def launch(self, stream: Optional[int] = None) -> None:
        if stream is None:
            stream = torch.cuda.current_stream(self.device).cuda_stream
        rc = _lib().rvq_persist_step(ctypes.c_void_p(self.plan.data_ptr()), ctypes.c_void_p(stream))
        if rc:
            _native.check(rc, "rvq_persist_step")

    @staticmethod
    def take_error() -> bool:
        """Whether a step since the last call gave up on a wait (its outputs
        are then invalid).  Synchronises the device."""
        rc = _lib().rvq_persist_take_error()
        if rc < 0:
            _native.check(-rc, "rvq_persist_take_error")
        return rc == 1
