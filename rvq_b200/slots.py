"""Ping-pong layer slots: flat arenas, a persistent decode stream, events.

Replaces the slot handling of the reference engines:

* ``_layerwise_logits`` in infer_compressed_layerwise_triton.py:240-294 makes
  new slot dicts and a new side stream on every call, ``torch.empty``s slot
  tensors inside ``with torch.cuda.stream(side)`` (249-262) and only makes the
  main stream wait for the side stream (272-274).  Nothing makes the side
  stream wait for the main stream, so refilling slot (l+1) % 2 can overwrite
  the weights layer l-1 is still reading (a write-after-read race).
* ``SlotResidency`` (infer_compressed_layerwise_single_slot.py:417-679) adds
  ready events (652-675) but releases a slot as soon as ``run_layer`` is
  *enqueued* (572-582, 902-906), with the same race.

Here:

* two flat device arenas, each sized for the largest layer (sum of
  ``numel * element_size`` of its decoded tensors, 256-byte aligned per
  tensor), allocated once; every layer decodes into views of arena l % 2;
* one persistent side stream; per slot a ``ready`` event (decode done, side
  -> main) and a ``free`` event (last forward that read the slot, main ->
  side).  A refill waits for ``free``, a forward waits for ``ready``;
* each layer's decode is one kernel launch (``LayerDecodePlan``), built once.

NVTX labels keep the reference's names (``layer_{i:03d}_decode_prefetch``,
``layer_{i:03d}_forward``; infer_compressed_layerwise_single_slot.py:661, 901).
"""

from __future__ import annotations

from contextlib import contextmanager
from dataclasses import dataclass
from typing import Dict, List, Sequence, Tuple

import torch

from .engine import LayerDecodePlan

ALIGN = 256


@dataclass(frozen=True)
class SlotSpec:
    """One decoded tensor of a layer: its name relative to the layer, shape, dtype."""
    rel_key: str
    shape: Tuple[int, ...]
    dtype: torch.dtype

    @property
    def nbytes(self) -> int:
        n = 1
        for s in self.shape:
            n *= int(s)
        return n * torch.empty((), dtype=self.dtype).element_size()


def aligned(n: int, a: int = ALIGN) -> int:
    return (n + a - 1) // a * a


def layout(specs: Sequence[SlotSpec]) -> Tuple[Dict[str, int], int]:
    """Byte offset of every tensor of one layer inside a slot, and the bytes used."""
    offsets, off = {}, 0
    for sp in specs:
        offsets[sp.rel_key] = off
        off += aligned(sp.nbytes)
    return offsets, off


def arena_bytes(layers: Sequence[Sequence[SlotSpec]]) -> int:
    """Slot size: the largest layer's laid-out bytes."""
    return max((layout(specs)[1] for specs in layers), default=0)


def relative_key(key: str, layer_idx: int) -> str:
    """Name of a tensor inside its layer (infer_compressed_layerwise_triton.py:253)."""
    return key.split(f"layers.{layer_idx}.")[-1]


def layer_specs_from_plan(plan, runtime_dtype: torch.dtype) -> List[List[SlotSpec]]:
    """Slot specs of every layer from the engine's layer plan
    (``_build_layer_plan``, infer_compressed_layerwise_triton.py:121-158)."""
    out = []
    for layer_idx, keys in enumerate(plan["layer_keys"]):
        specs = []
        for key in keys:
            entry = plan["entries"][key]
            specs.append(SlotSpec(relative_key(key, layer_idx), tuple(int(s) for s in entry["shape"]),
                                  runtime_dtype))
        out.append(specs)
    return out


class SlotArena:
    """``n_slots`` flat byte buffers and cached per-layer views into them."""

    def __init__(self, layers: Sequence[Sequence[SlotSpec]], device: torch.device, n_slots: int = 2):
        self.layers = [list(s) for s in layers]
        self.n_slots = n_slots
        self.nbytes = arena_bytes(self.layers)
        self.buffers = [torch.empty(max(self.nbytes, ALIGN), dtype=torch.uint8, device=device)
                        for _ in range(n_slots)]
        self._views: Dict[int, Dict[str, torch.Tensor]] = {}

    def slot_of(self, layer_idx: int) -> int:
        return layer_idx % self.n_slots

    def views(self, layer_idx: int) -> Dict[str, torch.Tensor]:
        v = self._views.get(layer_idx)
        if v is None:
            specs = self.layers[layer_idx]
            offsets, _ = layout(specs)
            buf = self.buffers[self.slot_of(layer_idx)]
            v = {}
            for sp in specs:
                off = offsets[sp.rel_key]
                v[sp.rel_key] = buf[off:off + sp.nbytes].view(sp.dtype).view(sp.shape)
            self._views[layer_idx] = v
        return v


@contextmanager
def nvtx_range(label: str):
    if torch.cuda.is_available():
        torch.cuda.nvtx.range_push(label)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield


class PingPongSlots:
    """Decode-ahead of layer l+1 into the other slot while layer l runs.

    Call order per forward pass (what ``_layerwise_logits`` does):

        slots.prefetch(0)                      # unless already pending
        for l in layers:
            w = slots.acquire(l)               # main waits for ready[l % 2]
            slots.prefetch(l + 1)              # side waits for free[(l+1) % 2]
            ... forward of layer l reading w ...
            slots.release(l)                   # free[l % 2] recorded on main
    """

    def __init__(self, plan, codebooks: Dict[str, torch.Tensor], device: torch.device,
                 runtime_dtype: torch.dtype):
        self.device = torch.device(device)
        self.runtime_dtype = runtime_dtype
        self.num_layers = len(plan["layer_keys"])
        self.arena = SlotArena(layer_specs_from_plan(plan, runtime_dtype), self.device)
        self.decode_plans: List[LayerDecodePlan] = []
        for layer_idx, keys in enumerate(plan["layer_keys"]):
            items = [(relative_key(k, layer_idx), plan["entries"][k]) for k in keys]
            self.decode_plans.append(LayerDecodePlan(items, codebooks, self.arena.views(layer_idx)))
        self.side = torch.cuda.Stream(self.device)
        self.ready = [torch.cuda.Event() for _ in range(self.arena.n_slots)]
        self.free = [torch.cuda.Event() for _ in range(self.arena.n_slots)]
        self.pending = set()
        self.launches = 0

    @property
    def slot_bytes(self) -> int:
        return self.arena.nbytes

    def prefetch(self, layer_idx: int) -> None:
        if layer_idx >= self.num_layers or layer_idx in self.pending:
            return
        s = self.arena.slot_of(layer_idx)
        with nvtx_range(f"layer_{layer_idx:03d}_decode_prefetch"):
            self.side.wait_event(self.free[s])          # last reader of this slot is done
            self.decode_plans[layer_idx].launch(self.side.cuda_stream)
            self.ready[s].record(self.side)
        self.launches += self.decode_plans[layer_idx].launches
        self.pending.add(layer_idx)

    def acquire(self, layer_idx: int, stream=None) -> Dict[str, torch.Tensor]:
        if layer_idx not in self.pending:
            self.prefetch(layer_idx)
        stream = stream or torch.cuda.current_stream(self.device)
        stream.wait_event(self.ready[self.arena.slot_of(layer_idx)])
        self.pending.discard(layer_idx)
        return self.arena.views(layer_idx)

    def release(self, layer_idx: int, stream=None) -> None:
        stream = stream or torch.cuda.current_stream(self.device)
        self.free[self.arena.slot_of(layer_idx)].record(stream)
