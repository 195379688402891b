"""GPU: the native pack loader (rvq_pack_load) delivers every tensor of the
artifact bit for bit, and a layer decoded from pack-loaded entries equals the
same layer decoded from the torch-loaded ones."""

import pytest
import torch

from rvq_b200 import pack, synthetic
from rvq_b200.engine import LayerDecodePlan

pytestmark = pytest.mark.gpu


def test_pack_load_matches_artifact(tmp_path, cuda_device):
    shape = synthetic.BlockShape(hidden=512, intermediate=1536, n_heads=8, n_kv_heads=2, head_dim=64)
    art = synthetic.make_model_artifact(shape, 3, 4096, seed=17)
    path = str(tmp_path / "m.rvqpack")
    pack.write_pack(art, path)
    got = pack.read_pack(path, cuda_device)
    torch.cuda.synchronize()
    for k, cb in art["shared_codebooks"].items():
        assert torch.equal(got["shared_codebooks"][k].cpu(), cb)
    for key, e in art["entries"].items():
        for f, v in e.items():
            if torch.is_tensor(v):
                assert got["entries"][key][f].dtype == v.dtype and torch.equal(got["entries"][key][f].cpu(), v), (key, f)
            else:
                assert got["entries"][key][f] == v, (key, f)
    # one layer decoded from both copies
    pre = "model.layers.1."
    items_pack = [(k[len(pre):], e) for k, e in got["entries"].items() if k.startswith(pre)]
    items_ref = [(k[len(pre):], {f: (v.to(cuda_device) if torch.is_tensor(v) else v) for f, v in e.items()})
                 for k, e in art["entries"].items() if k.startswith(pre)]
    cbs_p = {k: v.float() for k, v in got["shared_codebooks"].items()}
    cbs_r = {k: v.to(cuda_device, torch.float32) for k, v in art["shared_codebooks"].items()}
    outs_p = {n: torch.empty(tuple(e["shape"]), dtype=torch.bfloat16, device=cuda_device) for n, e in items_pack}
    outs_r = {n: torch.empty_like(t) for n, t in outs_p.items()}
    LayerDecodePlan(items_pack, cbs_p, outs_p).launch()
    LayerDecodePlan(items_ref, cbs_r, outs_r).launch()
    torch.cuda.synchronize()
    for n in outs_p:
        assert torch.equal(outs_p[n], outs_r[n]), n


def test_pack_load_errors(tmp_path, cuda_device):
    """A truncated pack is refused before any copy; the native loader refuses
    a byte range past the end of the file."""
    import ctypes
    from rvq_b200 import _native
    p = tmp_path / "short.rvqpack"
    art = {"format_version": 1, "entries": {"a": {"method": "bf16_raw", "data": torch.ones(5000, dtype=torch.bfloat16)}}}
    pack.write_pack(art, str(p))
    _, start, n = pack.read_header(str(p))
    buf = torch.empty(n + 8192, dtype=torch.uint8, device=cuda_device)
    lib = _native.load()
    pack.read_pack(str(p), cuda_device)                        # binds rvq_pack_load
    rc = lib.rvq_pack_load(str(p).encode(), start, n + 8192, ctypes.c_void_p(buf.data_ptr()), None)
    assert rc == _native.RVQ_ERR_INVALID
    p.write_bytes(p.read_bytes()[:-100])
    with pytest.raises(ValueError):
        pack.read_pack(str(p), cuda_device)
