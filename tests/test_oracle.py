"""The oracle pinned against the reference's own golden vectors (CPU only)."""

import numpy as np
import pytest

from oracle.c_oracle import decode_rvq_bits_c
from oracle.rvq_oracle import (OUT_BF16, OUT_F16, OUT_F32, RVQEntryNP, decode_rvq_bits, f32_to_bf16_bits,
                               f32_to_f16_bits)
from tests._golden import bits_equal, case_names, load_case

CASES = case_names()
KINDS = [OUT_F16, OUT_BF16, OUT_F32]


def test_golden_cases_present():
    assert len(CASES) >= 14, CASES


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("kind", KINDS)
def test_numpy_oracle_matches_reference(name, kind):
    case = load_case(name)
    got = decode_rvq_bits(case.entry_np(), kind)
    assert bits_equal(got, case.expected[kind], kind), name


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("kind", KINDS)
def test_c_oracle_matches_reference(name, kind):
    case = load_case(name)
    got = decode_rvq_bits_c(case.entry_np(), kind, nthreads=2)
    assert bits_equal(got, case.expected[kind], kind), name


def test_c_casts_match_numpy():
    from oracle import load_c_oracle
    lib = load_c_oracle()
    rng = np.random.default_rng(0)
    # every fp32 exponent, random mantissas, plus specials and rounding ties
    bitsu = rng.integers(0, 2**32, size=400_000, dtype=np.uint64).astype(np.uint32)
    special = np.array([0, 0x80000000, 0x7F800000, 0xFF800000, 0x477FEFFF, 0x477FF000,
                        0x477FE000, 0x33000000, 0x33000001, 0x38800000, 0x387FFFFF,
                        0x3F808000, 0x3F818000, 0x00000001, 0x7F7FFFFF], dtype=np.uint32)
    x = np.concatenate([bitsu, special]).view(np.float32)
    x = x[~np.isnan(x)]
    y16 = np.zeros(x.size, np.uint16)
    yb = np.zeros(x.size, np.uint16)
    lib.rvq_oracle_f32_to_f16(x.ctypes.data, y16.ctypes.data, x.size)
    lib.rvq_oracle_f32_to_bf16(x.ctypes.data, yb.ctypes.data, x.size)
    assert np.array_equal(y16, f32_to_f16_bits(x))
    assert np.array_equal(yb, f32_to_bf16_bits(x))


def test_bf16_cast_matches_torch():
    import torch
    rng = np.random.default_rng(1)
    x = rng.integers(0, 2**32, size=200_000, dtype=np.uint64).astype(np.uint32).view(np.float32)
    x = x[~np.isnan(x)]
    want = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(f32_to_bf16_bits(x), want)
    want16 = torch.from_numpy(x).to(torch.float16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(f32_to_f16_bits(x), want16)


def test_oracle_rejects_out_of_range_index():
    case = load_case("syn_k3_int16")
    e = case.entry_np()
    e.indices = e.indices.copy()
    e.indices[1, 5] = 600          # 512 codes
    with pytest.raises(IndexError):
        decode_rvq_bits(e, OUT_BF16)
    with pytest.raises(IndexError):
        decode_rvq_bits_c(e, OUT_BF16)


def test_planted_error_is_caught():
    """A mistake planted in the oracle's input must make the golden check fail."""
    case = load_case("enc_g128")
    e = case.entry_np()
    e.codebook = e.codebook.copy()
    e.codebook[2, 17, 3] += np.float32(1e-3)
    used = (case.indices[2] == 17).any()
    assert used
    got = decode_rvq_bits(e, OUT_F32)
    assert not bits_equal(got, case.expected[OUT_F32], OUT_F32)


def test_stage_order_is_sequential_from_positive_zero():
    """K <= 17: torch's stage sum equals an explicit left-to-right loop from +0.0,
    which is what both oracles implement."""
    import torch
    g = torch.Generator().manual_seed(3)
    for K in (1, 2, 4, 8, 16, 17):
        cb = torch.randn(K, 256, 8, generator=g)
        idx = torch.randint(0, 256, (K, 5000), generator=g)
        gathered = cb[torch.arange(K)[:, None], idx]
        acc = torch.zeros_like(gathered[0])
        for k in range(K):
            acc = acc + gathered[k]
        assert torch.equal(gathered.sum(0), acc), K


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("kind", KINDS)
def test_torch_port_matches_reference(name, kind):
    """The PyTorch restatement timed as the reference's own CPU baseline gives
    the reference's bits on every golden case."""
    import torch
    from oracle.torch_port import decode_rvq_into
    case = load_case(name)
    dt = {OUT_F16: torch.float16, OUT_BF16: torch.bfloat16, OUT_F32: torch.float32}[kind]
    out = torch.zeros(int(np.prod(case.meta["shape"])), dtype=dt)
    decode_rvq_into(case.entry_torch(), case.codebook_torch(dtype=torch.float32), out)
    bits = out.view(torch.int32 if kind == OUT_F32 else torch.int16).numpy()
    bits = bits.view(np.uint32 if kind == OUT_F32 else np.uint16)
    assert bits_equal(bits, case.expected[kind], kind), name


@pytest.mark.parametrize("name", __import__("tests._golden", fromlist=["int8_case_names"]).int8_case_names())
@pytest.mark.parametrize("kind", KINDS)
def test_int8_oracles_match_reference(name, kind):
    """numpy oracle and the PyTorch restatement of _decode_int8_into against
    the reference's own int8 golden output."""
    import torch
    from oracle.rvq_oracle import bf16_bits_to_f32, decode_int8_bits, f16_bits_to_f32
    from oracle.torch_port import decode_int8_into
    from tests._golden import load_int8_case
    case = load_int8_case(name)
    numel = int(np.prod(case.meta["shape"]))
    got = decode_int8_bits(case.q, f16_bits_to_f32(case.scales_f16), bf16_bits_to_f32(case.tail_bf16),
                           int(case.meta["group_size"]), numel, kind)
    assert bits_equal(got, case.expected[kind], kind), name
    dt = {OUT_F16: torch.float16, OUT_BF16: torch.bfloat16, OUT_F32: torch.float32}[kind]
    out = torch.zeros(numel, dtype=dt)
    decode_int8_into(case.entry_torch(), out)
    b = out.view(torch.int32 if kind == OUT_F32 else torch.int16).numpy()
    assert bits_equal(b.view(np.uint32 if kind == OUT_F32 else np.uint16), case.expected[kind], kind), name


@pytest.mark.parametrize("kind", KINDS)
def test_oracles_match_reference_at_projection_shape(kind):
    """The reference-encoded [1024, 2560] group-128 entry: the C oracle's
    decode hashes to the reference's own output."""
    import hashlib
    from oracle.rvq_oracle import f16_bits_to_f32
    from tests._golden import load_projection
    p = load_projection()
    ent = RVQEntryNP(indices=p["indices"], codebook=f16_bits_to_f32(p["codebook_f16"].view(np.uint16)),
                     scales=f16_bits_to_f32(p["scales_f16"].view(np.uint16)), tail=np.zeros(0, np.float32), d=8,
                     group_size=128, trimmed_numel=1024 * 2560, numel=1024 * 2560)
    got = decode_rvq_bits_c(ent, kind, nthreads=4)
    assert hashlib.sha256(got.tobytes()).hexdigest() == p["sha256"][kind]
