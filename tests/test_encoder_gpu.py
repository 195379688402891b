"""GPU: the encoder and k-means (rvq_b200/encoder.py) against the reference's
own compressor (golden vectors from tests/golden/make_golden_encoder.py).

The reference sums pairwise_sqdist's 8-term dot products in its CPU BLAS's
order, so the nearest code can only differ where the two best distances are
within fp32 rounding of each other; k-means is compared by the quality of
its centroids (and is deterministic run to run)."""

import os

import numpy as np
import pytest
import torch

from rvq_b200 import encoder

pytestmark = pytest.mark.gpu

CASES = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "encoder_cases.npz"))
TIE = 1e-5                     # distances within this are near-ties (fp32 rounding of ~1-unit distances)


def test_assign_codes_matches_reference(cuda_device):
    x = torch.from_numpy(CASES["assign_x"]).to(cuda_device)
    c = torch.from_numpy(CASES["assign_c"]).to(cuda_device)
    got = encoder.assign_codes(x, c, 4096).cpu().numpy()
    want, gap = CASES["assign_idx"], CASES["assign_gap"]
    diff = got != want
    assert not np.any(diff & (gap >= TIE)), np.nonzero(diff & (gap >= TIE))[0][:10]
    assert diff.mean() <= 1e-3


def test_kmeans_quality_and_determinism(cuda_device):
    x = torch.from_numpy(CASES["kmeans_x"]).to(cuda_device)
    a = encoder.kmeans_train(x, 64, 4, 7, 8192)
    b = encoder.kmeans_train(x, 64, 4, 7, 8192)
    assert torch.equal(a, b)
    idx = encoder.assign_codes(x, a)
    mse = float(((x - a[idx]) ** 2).sum(dim=1).mean())
    ref = float(CASES["kmeans_mse"])
    assert abs(mse - ref) <= 0.01 * ref, (mse, ref)


def test_encode_rvq_tensor_matches_reference(cuda_device):
    from oracle.rvq_oracle import OUT_BF16, RVQEntryNP, decode_rvq_bits
    from rvq_b200.engine import decode_into
    w = torch.from_numpy(CASES["enc_w"])
    cbs = torch.from_numpy(CASES["enc_codebooks"]).view(torch.float16).to(cuda_device)
    e = encoder.encode_rvq_tensor(w, cbs, 8, 128, 8192, "fixture")
    assert torch.equal(e["scales"].cpu().view(torch.int16), torch.from_numpy(CASES["enc_scales"]))
    codes = e["indices"].cpu().numpy()
    want = CASES["enc_codes"]
    assert codes.shape == want.shape and codes.dtype == want.dtype
    same = np.all(codes == want, axis=0)
    assert same.mean() >= 0.999, same.mean()
    ref = float(CASES["enc_rel_rmse"])
    assert abs(e["rel_rmse"] - ref) <= 1e-3 * ref, (e["rel_rmse"], ref)
    # the entry decodes on the GPU exactly as the oracle decodes it
    out = torch.empty(96, 512, dtype=torch.bfloat16, device=cuda_device)
    decode_into(e, {"fixture": cbs.float()}, out)
    torch.cuda.synchronize()
    ent = RVQEntryNP(indices=codes, codebook=cbs.float().cpu().numpy(), scales=e["scales"].float().cpu().numpy(),
                     tail=e["tail"].float().cpu().numpy(), d=8, group_size=128,
                     trimmed_numel=e["trimmed_numel"], numel=96 * 512)
    got = out.cpu().view(torch.int16).numpy().view(np.uint16).reshape(-1)
    assert np.array_equal(got, decode_rvq_bits(ent, OUT_BF16))
