"""Slot sizing and layout (host logic, CPU)."""

import torch

from rvq_b200.slots import ALIGN, SlotArena, SlotSpec, arena_bytes, layout, relative_key


def specs(n_layers, sizes):
    return [[SlotSpec(f"t{i}", (s,), torch.bfloat16) for i, s in enumerate(sizes)] for _ in range(n_layers)]


def test_layout_is_aligned_and_disjoint():
    sp = [SlotSpec("a", (3, 5), torch.bfloat16), SlotSpec("b", (7,), torch.float32),
          SlotSpec("c", (128, 64), torch.bfloat16)]
    offs, total = layout(sp)
    assert all(o % ALIGN == 0 for o in offs.values())
    ranges = sorted((offs[s.rel_key], offs[s.rel_key] + s.nbytes) for s in sp)
    assert all(r0[1] <= r1[0] for r0, r1 in zip(ranges, ranges[1:]))
    assert total == ranges[-1][1] + (-ranges[-1][1]) % ALIGN


def test_arena_is_sized_for_the_largest_layer():
    layers = specs(2, [100, 2000]) + [[SlotSpec("big", (10000,), torch.bfloat16)]]
    assert arena_bytes(layers) == 20000 // ALIGN * ALIGN + (ALIGN if 20000 % ALIGN else 0)
    arena = SlotArena(layers, torch.device("cpu"))
    assert len(arena.buffers) == 2 and arena.buffers[0].numel() == arena.nbytes
    v0, v1 = arena.views(0), arena.views(1)
    assert v0["t1"].data_ptr() != v1["t1"].data_ptr()           # layers 0, 1 use different slots
    assert arena.views(2)["big"].data_ptr() == arena.buffers[0].data_ptr()
    assert v0["t1"].shape == (2000,) and v0["t1"].dtype == torch.bfloat16


def test_relative_key():
    assert relative_key("model.layers.12.mlp.up_proj.weight", 12) == "mlp.up_proj.weight"
    assert relative_key("model.layers.1.self_attn.q_norm.weight", 1) == "self_attn.q_norm.weight"
