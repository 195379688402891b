#!/usr/bin/env python3
"""Golden end-to-end vectors from the reference's own layerwise engine.

Runs ``_layerwise_logits`` of infer_compressed_layerwise_triton.py (engine A)
on the CPU over a tiny random Qwen3 model stored as a synthetic RVQ artifact,
then greedy-decodes a few tokens with the token loop of its
``generate_greedy`` (lines 323-386, on token ids instead of text).  Writes
``engine_tiny.npz``: prompt, generated ids and every step's logits.

Run where a checkout of the reference is available, giving its path:

    python tests/golden/make_golden_engine.py <reference checkout>
    (or RVQ_REFERENCE_DIR=<reference checkout> python tests/golden/make_golden_engine.py)

The reference engine needs ``accelerate`` (absent here) and CUDA streams;
this script provides, for the CPU run only:
* an ``accelerate`` stand-in with ``init_empty_weights`` (parameters created
  on the meta device, buffers kept) and ``set_module_tensor_to_device``;
* no-op stand-ins for ``torch.cuda.Stream``/``stream``/``current_stream``;
* the reference's own CPU decode ``_decode_rvq_into``
  (infer_compressed_layerwise_single_slot.py:123-149) behind the engine's
  ``decode_rvq_triton_into`` name.
"""

from __future__ import annotations

import contextlib
import os
import sys
import tempfile
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("RVQ_REFERENCE_DIR") or (sys.argv[1] if len(sys.argv) > 1 else "")
if not REF or not os.path.isdir(REF):
    sys.exit(f"usage: {os.path.basename(__file__)} <reference checkout> (or set RVQ_REFERENCE_DIR)")
sys.path.insert(0, REF)
sys.path.insert(0, REPO)

import transformers  # noqa: E402,F401  (import before the accelerate stand-in)

from rvq_b200 import synthetic  # noqa: E402

TINY = synthetic.BlockShape(hidden=64, intermediate=128, n_heads=4, n_kv_heads=2, head_dim=16)
N_LAYERS, VOCAB, SEED = 2, 512, 5
PROMPT_LEN, NEW_TOKENS = 12, 6


def install_accelerate_stub():
    acc = types.ModuleType("accelerate")
    utils = types.ModuleType("accelerate.utils")
    modeling = types.ModuleType("accelerate.utils.modeling")

    @contextlib.contextmanager
    def init_empty_weights():
        orig = torch.nn.Module.register_parameter

        def register(self, name, param):
            orig(self, name, param)
            if param is not None:
                p = self._parameters[name]
                self._parameters[name] = torch.nn.Parameter(p.to("meta"), requires_grad=p.requires_grad)
        torch.nn.Module.register_parameter = register
        try:
            yield
        finally:
            torch.nn.Module.register_parameter = orig

    def set_module_tensor_to_device(module, tensor_name, device, value=None, dtype=None):
        parts = tensor_name.split(".")
        for part in parts[:-1]:
            module = getattr(module, part)
        name = parts[-1]
        if value is None:
            value = getattr(module, name)
        value = value.to(device)
        if dtype is not None and value.is_floating_point():
            value = value.to(dtype)
        if name in module._parameters:
            module._parameters[name] = torch.nn.Parameter(value, requires_grad=False)
        else:
            module._buffers[name] = value

    acc.init_empty_weights = init_empty_weights
    modeling.set_module_tensor_to_device = set_module_tensor_to_device
    utils.modeling = modeling
    acc.utils = utils
    sys.modules["accelerate"] = acc
    sys.modules["accelerate.utils"] = utils
    sys.modules["accelerate.utils.modeling"] = modeling


class _NoStream:
    def __init__(self, *a, **k):
        pass

    def wait_stream(self, other):
        pass


def install_cpu_streams():
    torch.cuda.Stream = _NoStream
    torch.cuda.stream = lambda s: contextlib.nullcontext()
    torch.cuda.current_stream = lambda device=None: _NoStream()


def run_reference(artifact, runtime_dtype=torch.bfloat16):
    install_accelerate_stub()
    install_cpu_streams()
    import infer_compressed_layerwise_single_slot as ss
    import infer_compressed_layerwise_triton as eng
    ss.torch = torch
    eng.rvq_triton_supported = lambda entry, out: True
    eng.decode_rvq_triton_into = lambda entry, cb, out: ss._decode_rvq_into(entry, cb, out)

    device = torch.device("cpu")
    cfg = synthetic.qwen3_config(TINY, N_LAYERS, VOCAB)
    with tempfile.TemporaryDirectory() as d:
        cfg.save_pretrained(d)
        model = eng._build_meta_model(d)
    gpu_codebooks = {k: v.to(device, dtype=torch.float32) for k, v in artifact["shared_codebooks"].items()}
    gpu_entries = {k: dict(v) for k, v in artifact["entries"].items()}
    plan = eng._build_layer_plan(model, gpu_entries)
    embed = eng.decode_to_tensor(plan["entries"][plan["embed_key"]], gpu_codebooks, device, runtime_dtype)
    lm_head = embed if plan["lm_head_key"] is None else eng.decode_to_tensor(
        plan["entries"][plan["lm_head_key"]], gpu_codebooks, device, runtime_dtype)
    from accelerate.utils.modeling import set_module_tensor_to_device
    for key in plan["norm_keys"]:
        val = eng.decode_to_tensor(plan["entries"][key], gpu_codebooks, device, runtime_dtype)
        set_module_tensor_to_device(model, key, device, value=val, dtype=runtime_dtype)

    gen = torch.Generator().manual_seed(SEED + 1)
    prompt = torch.randint(0, VOCAB, (1, PROMPT_LEN), generator=gen)
    generated = prompt
    attention = torch.ones_like(prompt)
    cache = eng._make_dynamic_cache(plan["base_model"])
    steps = []
    with torch.inference_mode():
        logits, cache = eng._layerwise_logits(model, plan, gpu_codebooks, embed, lm_head, generated,
                                              attention, cache, torch.arange(PROMPT_LEN), device,
                                              runtime_dtype)
        cache.has_previous_state = True
        steps.append(logits.float().numpy())
        for _ in range(NEW_TOKENS):
            nxt = logits.argmax(dim=-1, keepdim=True)
            generated = torch.cat([generated, nxt], dim=1)
            attention = torch.cat([attention, torch.ones_like(nxt)], dim=1)
            logits, cache = eng._layerwise_logits(model, plan, gpu_codebooks, embed, lm_head, nxt,
                                                  attention, cache,
                                                  torch.tensor([generated.shape[1] - 1]), device,
                                                  runtime_dtype)
            steps.append(logits.float().numpy())
    return prompt.numpy(), generated[:, PROMPT_LEN:].numpy(), np.stack(steps)


def main():
    artifact = synthetic.make_model_artifact(TINY, N_LAYERS, VOCAB, seed=SEED)
    prompt, gen_ids, logits = run_reference(artifact)
    np.savez_compressed(os.path.join(HERE, "engine_tiny.npz"), prompt=prompt, generated=gen_ids,
                        logits=logits, n_layers=N_LAYERS, vocab=VOCAB, seed=SEED)
    print("prompt", prompt.tolist())
    print("generated", gen_ids.tolist())
    print("logits", logits.shape, float(np.abs(logits).max()))


if __name__ == "__main__":
    main()
