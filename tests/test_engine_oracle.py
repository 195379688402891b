"""The engine oracle pinned against the reference engine's own end-to-end
output (tests/golden/engine_tiny.npz), on the CPU."""

import os

import numpy as np
import torch

from oracle.engine_ref import OracleEngine
from rvq_b200 import synthetic

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "engine_tiny.npz")
TINY = synthetic.BlockShape(hidden=64, intermediate=128, n_heads=4, n_kv_heads=2, head_dim=16)


def load():
    z = np.load(GOLDEN)
    return z, int(z["n_layers"]), int(z["vocab"]), int(z["seed"])


def test_oracle_engine_matches_reference_engine_on_cpu():
    z, n_layers, vocab, seed = load()
    art = synthetic.make_model_artifact(TINY, n_layers, vocab, seed=seed)
    cfg = synthetic.qwen3_config(TINY, n_layers, vocab)
    eng = OracleEngine(cfg, art, "cpu", torch.bfloat16)
    prompt = torch.from_numpy(z["prompt"])
    gen, steps = eng.generate(prompt, z["generated"].shape[1])
    assert np.array_equal(gen.numpy(), z["generated"])
    got = np.stack([s.float().numpy() for s in steps])
    assert np.array_equal(got, z["logits"])
