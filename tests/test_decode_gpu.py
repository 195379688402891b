"""GPU parity of the sm_100a decode against the reference's own outputs.

Bar: bit-exact (NaN payloads excepted) for every golden case, output dtype
and codebook dtype; full-size workloads checked by sha256 against the
reference's result; random larger cases against the C oracle.
"""

import hashlib

import numpy as np
import pytest
import torch

from oracle.c_oracle import decode_rvq_bits_c
from oracle.rvq_oracle import OUT_BF16, OUT_F16, OUT_F32, RVQEntryNP
from rvq_b200 import _native, synthetic
from rvq_b200.triton_decode_kernels import decode_rvq_triton_into, rvq_triton_supported
from tests._golden import bits_equal, case_names, load_case, load_checksums

pytestmark = pytest.mark.gpu

CASES = case_names()
KINDS = {OUT_F16: torch.float16, OUT_BF16: torch.bfloat16, OUT_F32: torch.float32}


def out_bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.float32:
        return t.view(torch.int32).numpy().view(np.uint32).reshape(-1)
    return t.view(torch.int16).numpy().view(np.uint16).reshape(-1)


def entry_np_from_torch(entry, cb) -> RVQEntryNP:
    numel = int(np.prod(entry["shape"]))
    return RVQEntryNP(indices=entry["indices"].cpu().numpy(), codebook=cb.float().cpu().numpy(),
                      scales=entry["scales"].float().cpu().numpy(),
                      tail=entry["tail"].float().cpu().numpy(), d=int(entry["d"]),
                      group_size=int(entry["group_size"]),
                      trimmed_numel=int(entry["trimmed_numel"]), numel=numel)


@pytest.mark.parametrize("cb_dtype", ["f16", "f32"])
@pytest.mark.parametrize("kind", list(KINDS))
@pytest.mark.parametrize("name", CASES)
def test_golden_bit_exact(name, kind, cb_dtype, cuda_device):
    case = load_case(name)
    entry = case.entry_torch(cuda_device)
    cb = case.codebook_torch(cuda_device)
    if cb_dtype == "f32":
        cb = cb.to(torch.float32)
    elif cb.dtype != torch.float16:
        pytest.skip("fp32-only codebook")
    out = torch.zeros(tuple(case.meta["shape"]), dtype=KINDS[kind], device=cuda_device)
    assert rvq_triton_supported(entry, out)
    ret = decode_rvq_triton_into(entry, cb, out)
    assert ret is out
    torch.cuda.synchronize()
    assert bits_equal(out_bits(out), case.expected[kind], kind), name


@pytest.mark.parametrize("name", ["enc_tail", "syn_trimmed_short", "syn_ragged_tail"])
def test_untouched_beyond_written_range(name, cuda_device):
    """Only out[:trimmed + tail] is written (triton_decode_kernels.py:104, 187-188)."""
    case = load_case(name)
    entry = case.entry_torch(cuda_device)
    cb = case.codebook_torch(cuda_device, torch.float32)
    numel = int(np.prod(case.meta["shape"]))
    big = torch.full((numel + 37,), 7.0, dtype=torch.bfloat16, device=cuda_device)
    out = big[:numel].view(tuple(case.meta["shape"]))
    decode_rvq_triton_into(entry, cb, out)
    torch.cuda.synchronize()
    written = case.meta["trimmed_numel"] + int(case.tail_bf16.size)
    assert bits_equal(out_bits(out)[:written], case.expected[OUT_BF16][:written], OUT_BF16)
    assert torch.all(big[written:] == 7.0)


@pytest.mark.parametrize("kind", list(KINDS))
def test_misaligned_output_view(kind, cuda_device):
    case = load_case("enc_g128")
    entry = case.entry_torch(cuda_device)
    cb = case.codebook_torch(cuda_device, torch.float32)
    numel = int(np.prod(case.meta["shape"]))
    base = torch.zeros(numel + 1, dtype=KINDS[kind], device=cuda_device)
    out = base[1:].view(tuple(case.meta["shape"]))      # 2- or 4-byte offset
    assert out.data_ptr() % 16 != 0
    decode_rvq_triton_into(entry, cb, out)
    torch.cuda.synchronize()
    assert bits_equal(out_bits(out), case.expected[kind], kind)


def test_side_stream_then_event(cuda_device):
    case = load_case("enc_rowscale")
    entry = case.entry_torch(cuda_device)
    cb = case.codebook_torch(cuda_device, torch.float32)
    out = torch.zeros(tuple(case.meta["shape"]), dtype=torch.bfloat16, device=cuda_device)
    side = torch.cuda.Stream(cuda_device)
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        decode_rvq_triton_into(entry, cb, out)
        ready = torch.cuda.Event()
        ready.record(side)
    torch.cuda.current_stream().wait_event(ready)
    got = out.clone()
    torch.cuda.synchronize()
    assert bits_equal(out_bits(got), case.expected[OUT_BF16], OUT_BF16)


@pytest.mark.parametrize("seed,shape,group,stages,ncodes", [
    (1, (1000, 768), 128, 4, 256),
    (2, (333, 520), 520, 4, 256),
    (3, (2048, 1024), 64, 3, 256),
    (4, (517, 96), 96, 4, 1024),         # int16 indices, 1024 codes
    (5, (64, 4096), 4096, 6, 256),       # K=6 (generic stage loop)
    (6, (128, 512), 16, 2, 64),          # 64 codes in uint8 indices
])
@pytest.mark.parametrize("cb_dtype", [torch.float16, torch.float32])
def test_random_vs_c_oracle(seed, shape, group, stages, ncodes, cb_dtype, cuda_device):
    g = torch.Generator().manual_seed(seed)
    cb = synthetic.make_codebook(stages, ncodes, 8, g)
    entry = synthetic.make_rvq_entry(shape[0], shape[1], g, stages=stages, ncodes=ncodes,
                                     group_size=group)
    want = decode_rvq_bits_c(entry_np_from_torch(entry, cb), OUT_BF16)
    dev_entry = {k: (v.to(cuda_device) if torch.is_tensor(v) else v) for k, v in entry.items()}
    out = torch.empty(shape, dtype=torch.bfloat16, device=cuda_device)
    decode_rvq_triton_into(dev_entry, cb.to(cuda_device, cb_dtype), out)
    torch.cuda.synchronize()
    assert bits_equal(out_bits(out), want, OUT_BF16)
    assert not _native.take_index_error()


def test_config0_full_size_checksum(cuda_device):
    """[9728, 2560], K=4, per-row scales, fp16 out: sha256 of the reference's result."""
    entry, cb = synthetic.make_config0_entry(seed=0)
    dev = {k: (v.to(cuda_device) if torch.is_tensor(v) else v) for k, v in entry.items()}
    out = torch.empty(tuple(entry["shape"]), dtype=torch.float16, device=cuda_device)
    decode_rvq_triton_into(dev, cb.to(cuda_device, torch.float32), out)
    digest = hashlib.sha256(out_bits(out).tobytes()).hexdigest()
    assert digest == load_checksums()["config0_seed0_f16"]


def test_block_layer_launch_checksums(cuda_device):
    """All 7 projections + 4 norms of one 2560/9728 block in ONE launch."""
    from rvq_b200.engine import LayerDecodePlan
    art = synthetic.make_block_artifact(seed=0)
    cbs = {k: v.to(cuda_device, torch.float32) for k, v in art["shared_codebooks"].items()}
    entries = {k: {ek: (ev.to(cuda_device) if torch.is_tensor(ev) else ev) for ek, ev in e.items()}
               for k, e in art["entries"].items()}
    outs = {k: torch.empty(tuple(e["shape"]), dtype=torch.bfloat16, device=cuda_device)
            for k, e in entries.items()}
    plan = LayerDecodePlan(list(entries.items()), cbs, outs)
    plan.launch(torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    sums = load_checksums()
    n_rvq = 0
    for key, e in entries.items():
        if e["method"] == "bf16_raw":
            assert torch.equal(outs[key].view(torch.int16), e["data"].view(torch.int16)), key
            continue
        n_rvq += 1
        digest = hashlib.sha256(out_bits(outs[key]).tobytes()).hexdigest()
        assert digest == sums[f"block_seed0_bf16:{key}"], key
    assert n_rvq == 7


def test_out_of_range_index_sets_flag(cuda_device):
    """An index >= ncodes is caught by the kernel's own bounds check: no
    out-of-bounds read, the sticky flag reports it."""
    g = torch.Generator().manual_seed(9)
    cb = synthetic.make_codebook(4, 16, 8, g)             # 16 codes, uint8 indices
    entry = synthetic.make_rvq_entry(64, 64, g, ncodes=16, group_size=64)
    entry["indices"][2, 5] = 200
    dev = {k: (v.to(cuda_device) if torch.is_tensor(v) else v) for k, v in entry.items()}
    out = torch.empty((64, 64), dtype=torch.bfloat16, device=cuda_device)
    _native.take_index_error()
    decode_rvq_triton_into(dev, cb.to(cuda_device), out)
    assert _native.take_index_error() is True
    assert _native.take_index_error() is False           # cleared by the read


def test_reference_exceptions(cuda_device):
    case = load_case("enc_g128")
    entry = case.entry_torch(cuda_device)
    cb = case.codebook_torch(cuda_device)
    out = torch.empty(tuple(case.meta["shape"]), dtype=torch.bfloat16, device=cuda_device)
    with pytest.raises(NotImplementedError):
        decode_rvq_triton_into(dict(entry, d=4), cb, out)
    with pytest.raises(ValueError):
        decode_rvq_triton_into(dict(entry, group_size=100), cb, out)
    with pytest.raises(ValueError):
        decode_rvq_triton_into(entry, cb, out.cpu())
    with pytest.raises(ValueError):
        decode_rvq_triton_into(entry, cb, out.t())
    with pytest.raises(ValueError):
        decode_rvq_triton_into(dict(entry, indices=entry["indices"].cpu()), cb, out)
    with pytest.raises(NotImplementedError):
        decode_rvq_triton_into(entry, cb, out.to(torch.int32))


def test_layer_launch_many_mixed_entries(cuda_device):
    """One launch, 25 RVQ entries of very different sizes (1 tile .. ~100 tiles,
    K = 1..4, int16 codes, tails) plus raw copies: the per-CTA job schedule
    must give every entry exactly the reference's result."""
    from rvq_b200.engine import LayerDecodePlan
    g = torch.Generator().manual_seed(77)
    items, cbs, outs, wants = [], {}, {}, {}
    shapes = [(8, 8), (64, 64), (3, 40), (500, 256), (1000, 96), (17, 8), (256, 512), (2, 1024)]
    for i in range(25):
        o, inn = shapes[i % len(shapes)]
        stages = [4, 4, 3, 2, 1, 4][i % 6]
        ncodes = 512 if i % 7 == 3 else 256
        group = [inn, 8, 64, inn][i % 4] if inn % 64 == 0 else inn
        if (o * inn) % 8:
            continue
        cb = synthetic.make_codebook(stages, ncodes, 8, g)
        e = synthetic.make_rvq_entry(o, inn, g, stages=stages, ncodes=ncodes, group_size=group,
                                     codebook_id=f"cb{i}")
        wants[f"e{i}"] = decode_rvq_bits_c(entry_np_from_torch(e, cb), OUT_BF16)
        cbs[f"cb{i}"] = cb.to(cuda_device, torch.float32 if i % 2 else torch.float16)
        items.append((f"e{i}", {k: (v.to(cuda_device) if torch.is_tensor(v) else v) for k, v in e.items()}))
        outs[f"e{i}"] = torch.empty((o, inn), dtype=torch.bfloat16, device=cuda_device)
    for i in range(4):
        data = torch.randn(300 + 7 * i, generator=g).to(torch.bfloat16)
        key = f"norm{i}"
        items.append((key, synthetic.make_raw_entry(data) | {"data": data.to(cuda_device)}))
        outs[key] = torch.empty(data.shape, dtype=torch.bfloat16, device=cuda_device)
        wants[key] = data.view(torch.int16).numpy().view(np.uint16)
    plan = LayerDecodePlan(items, cbs, outs)
    assert plan.launches == 1
    plan.launch()
    torch.cuda.synchronize()
    for key, want in wants.items():
        assert bits_equal(out_bits(outs[key]), want, OUT_BF16), key


@pytest.mark.parametrize("kind", list(KINDS))
def test_projection_shape_group128_matches_reference_hash(kind, cuda_device):
    """The reference-encoded [1024, 2560] entry at the compressor's default
    group size 128: the single-entry API (artifact planes) and, for bf16, the
    layer plan's slot kernel (quad codes) hash to the reference's output."""
    import hashlib
    from rvq_b200.engine import LayerDecodePlan
    from tests._golden import load_projection
    p = load_projection()
    cb = torch.from_numpy(p["codebook_f16"]).view(torch.float16).to(cuda_device).float()
    entry = {"method": "rvq_groupwise", "codebook_id": "attn_k_proj", "shape": [1024, 2560], "dtype": "bfloat16",
             "group_size": 128, "d": 8, "trimmed_numel": 1024 * 2560,
             "scales": torch.from_numpy(p["scales_f16"]).view(torch.float16).to(cuda_device),
             "indices": torch.from_numpy(p["indices"]).to(cuda_device),
             "tail": torch.zeros(0, dtype=torch.bfloat16, device=cuda_device)}
    out = torch.zeros(1024, 2560, dtype=KINDS[kind], device=cuda_device)
    decode_rvq_triton_into(entry, cb, out)
    torch.cuda.synchronize()
    assert hashlib.sha256(out_bits(out).tobytes()).hexdigest() == p["sha256"][kind]
    if KINDS[kind] == torch.bfloat16:
        slot = torch.zeros_like(out)
        LayerDecodePlan([("k", entry)], {"attn_k_proj": cb}, {"k": slot}).launch()
        torch.cuda.synchronize()
        assert hashlib.sha256(out_bits(slot).tobytes()).hexdigest() == p["sha256"][kind]
