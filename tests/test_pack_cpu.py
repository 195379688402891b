"""Artifact pack format (rvq_b200/pack.py) on the CPU: the header round-trips
every non-tensor field, and every tensor's bytes sit at its recorded,
page-aligned offset of the data region."""

import json

import numpy as np
import torch

from rvq_b200 import pack, synthetic


def test_pack_layout_round_trip(tmp_path):
    shape = synthetic.BlockShape(hidden=256, intermediate=512, n_heads=4, n_kv_heads=2, head_dim=64)
    art = synthetic.make_model_artifact(shape, 2, 512, seed=9)
    art["entries"]["model.layers.0.self_attn.q_proj.weight"]["note"] = {"nested": [1, 2.5, "x"]}
    path = str(tmp_path / "model.rvqpack")
    size = pack.write_pack(art, path)
    header, data_start, nbytes = pack.read_header(path)
    assert data_start % pack.ALIGN == 0 and data_start + nbytes == size
    raw = np.fromfile(path, dtype=np.uint8)[data_start:]

    def check(orig, desc):
        if torch.is_tensor(orig):
            off, n = desc["__tensor__"]
            assert off % pack.ALIGN == 0
            assert desc["dtype"] == pack._NAMES[orig.dtype] and desc["shape"] == list(orig.shape)
            want = orig.contiguous().view(torch.uint8).reshape(-1).numpy()
            assert np.array_equal(raw[off:off + n], want)
        elif isinstance(orig, dict):
            assert set(desc) == {str(k) for k in orig}
            for k, v in orig.items():
                check(v, desc[str(k)])
        else:
            assert json.loads(json.dumps(orig)) == desc

    check(art, header)


def test_rejects_truncated_pack(tmp_path):
    p = tmp_path / "t.rvqpack"
    pack.write_pack({"x": torch.arange(3000, dtype=torch.int32)}, str(p))
    p.write_bytes(p.read_bytes()[:-10])
    try:
        pack.read_header(str(p))
    except ValueError:
        return
    raise AssertionError("read_header accepted a truncated pack")


def test_rejects_foreign_file(tmp_path):
    p = tmp_path / "x.bin"
    p.write_bytes(b"not a pack at all")
    try:
        pack.read_header(str(p))
    except ValueError:
        return
    raise AssertionError("read_header accepted a foreign file")
