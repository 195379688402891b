"""GPU: native int8_groupwise decode against the reference's own golden output.

The fixtures (tests/golden/int8_*.npz, made by make_golden_int8.py) hold
entries from the reference's encode_int8_groupwise and the outputs of its
_decode_int8_into; the GPU path must reproduce them bit for bit (any NaN
equals any NaN) for fp16, bf16 and fp32 outputs, alone, at odd output
offsets, and mixed into one layer launch with RVQ entries and raw copies.
"""

import numpy as np
import pytest
import torch

from oracle.rvq_oracle import OUT_BF16, OUT_F16, OUT_F32
from rvq_b200.engine import LayerDecodePlan, decode_into
from tests._golden import bits_equal, int8_case_names, load_case, load_int8_case

pytestmark = pytest.mark.gpu

KINDS = {OUT_F16: torch.float16, OUT_BF16: torch.bfloat16, OUT_F32: torch.float32}


def out_bits(t, kind):
    b = t.cpu().contiguous().view(torch.int32 if kind == OUT_F32 else torch.int16).numpy()
    return b.view(np.uint32 if kind == OUT_F32 else np.uint16).reshape(-1)


@pytest.mark.parametrize("name", int8_case_names())
@pytest.mark.parametrize("kind", list(KINDS))
def test_int8_decode_matches_reference(name, kind, cuda_device):
    case = load_int8_case(name)
    entry = case.entry_torch(cuda_device)
    out = torch.full(tuple(case.meta["shape"]), float("nan"), dtype=KINDS[kind], device=cuda_device)
    decode_into(entry, {}, out)
    torch.cuda.synchronize()
    assert bits_equal(out_bits(out, kind), case.expected[kind], kind), name


@pytest.mark.parametrize("offset", [1, 3, 8])
def test_int8_misaligned_output_and_untouched_bytes(offset, cuda_device):
    """Output starting off a 16-byte boundary takes the element path; nothing
    past trimmed + tail is written."""
    case = load_int8_case("int8_big")
    entry = case.entry_torch(cuda_device)
    numel = int(np.prod(case.meta["shape"]))
    buf = torch.full((numel + offset + 64,), 7.0, dtype=torch.bfloat16, device=cuda_device)
    out = buf[offset:offset + numel]
    decode_into(entry, {}, out)
    torch.cuda.synchronize()
    assert bits_equal(out_bits(out, OUT_BF16), case.expected[OUT_BF16], OUT_BF16)
    assert torch.all(buf[:offset] == 7.0) and torch.all(buf[offset + numel:] == 7.0)


def test_int8_in_a_mixed_layer_launch(cuda_device):
    """int8 entries, RVQ entries and a raw copy in one rvq_decode_layer_mixed launch."""
    keys, items, outs, want = [], [], {}, {}
    for name in ("int8_g128", "int8_tail", "int8_g7"):
        c = load_int8_case(name)
        items.append((name, c.entry_torch(cuda_device)))
        outs[name] = torch.zeros(tuple(c.meta["shape"]), dtype=torch.bfloat16, device=cuda_device)
        want[name] = c.expected[OUT_BF16]
    cbs = {}
    for name in ("enc_g128", "syn_ragged_tail"):
        c = load_case(name)
        e = c.entry_torch(cuda_device)
        e["codebook_id"] = name
        cbs[name] = c.codebook_torch(cuda_device, torch.float32)
        items.append((name, e))
        outs[name] = torch.zeros(tuple(c.meta["shape"]), dtype=torch.bfloat16, device=cuda_device)
        want[name] = c.expected[OUT_BF16]
    raw = torch.randn(1000, device=cuda_device).to(torch.bfloat16)
    items.append(("norm", {"method": "bf16_raw", "shape": [1000], "dtype": "bfloat16", "data": raw}))
    outs["norm"] = torch.zeros(1000, dtype=torch.bfloat16, device=cuda_device)
    plan = LayerDecodePlan(items, cbs, outs)
    assert plan.launches == 1
    plan.launch()
    torch.cuda.synchronize()
    for name, w in want.items():
        assert bits_equal(out_bits(outs[name], OUT_BF16), w, OUT_BF16), name
    assert torch.equal(outs["norm"], raw)
