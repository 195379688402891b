"""Layerwise RVQ engine on B200: the drop-in ``_layerwise_logits``.

Same signature, arguments and results as the reference engine's
``_layerwise_logits`` (infer_compressed_layerwise_triton.py:202-298).  What
changes is how the slot weights get there: a persistent ``PingPongSlots``
(rvq_b200/slots.py) kept with the layer plan decodes each layer with ONE
kernel launch on a side stream, guarded by ready/free events, and starts
decoding layer 0 of the next call while the current call finishes.

The model math is untouched: each HF decoder layer runs through
``functional_call`` on the slot tensors exactly as in the reference
(lines 279-294), including the reference's choice of attention mask
(lines 223-238).

The set-up helpers below serve tests and benchmarks on synthetic artifacts
(the deployment keeps its own host set-up): a parameters-on-meta model (the
role accelerate's ``init_empty_weights`` plays in the reference), a layer
plan from the model's module tree, the artifact upload (lines 423-433) and
the always-resident tensors (lines 439-461).
"""

from __future__ import annotations

import contextlib
from typing import Dict, List, Optional

import torch
import torch.nn.functional as F

from .engine import decode_to_tensor
from .slots import PingPongSlots, nvtx_range

try:
    from torch.func import functional_call
except ImportError:  # pragma: no cover
    from torch.nn.utils.stateless import functional_call

_SLOTS_KEY = "_rvq_b200_slots"


# ---------------------------------------------------------------------------
# model / plan set-up
# ---------------------------------------------------------------------------

@contextlib.contextmanager
def params_on_meta():
    """Create module parameters on the meta device, buffers where they are.

    Parameters are replaced by slot tensors at call time, so they never need
    storage; buffers (the rotary ``inv_freq``) keep real values.  This is the
    behaviour the reference gets from accelerate's ``init_empty_weights``.
    """
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


def build_meta_model(config):
    """Qwen3 causal LM with parameters on meta and eager attention
    (infer_compressed_layerwise_triton.py:64-73)."""
    from transformers import AutoModelForCausalLM
    if hasattr(config, "_attn_implementation"):
        config._attn_implementation = "eager"
    with params_on_meta():
        model = AutoModelForCausalLM.from_config(config)
    return model.eval()


def plan_from_module_tree(model, entries: Dict[str, Dict[str, object]]):
    """The layer plan ``_layerwise_logits`` reads, for an artifact whose keys
    are the model's own parameter names (what this package's synthetic
    artifacts write).  In a deployment the engine's own plan builder hands the
    plan in; the drop-in forward only reads these keys of it: ``base_model``,
    ``entries``, ``layer_keys`` (per decoder layer, sorted), ``embed_key``,
    ``lm_head_key`` and ``norm_keys``.

    Built by walking the decoder's module tree: every parameter of decoder
    layer i, named by its path from the top-level model, that the artifact
    holds.  Artifacts written under another naming prefix need the
    deployment's plan builder, not this helper."""
    decoder = model.get_decoder()
    path = {id(m): name for name, m in model.named_modules()}

    def full(module, pname: str) -> str:
        base = path[id(module)]
        return f"{base}.{pname}" if base else pname

    layer_keys = []
    for layer in decoder.layers:
        keys = [full(layer, pname) for pname, _ in layer.named_parameters()]
        layer_keys.append(sorted(k for k in keys if k in entries))
    embed_key = full(decoder.embed_tokens, "weight")
    head = model.get_output_embeddings()
    lm_head_key = full(head, "weight") if head is not None else None
    norm_keys = sorted(full(decoder.norm, pname) for pname, _ in decoder.norm.named_parameters())
    held = lambda k: k if k is not None and k in entries else None
    return {
        "base_model": decoder,
        "entries": entries,
        "layer_keys": layer_keys,
        "embed_key": held(embed_key),
        "lm_head_key": held(lm_head_key),
        "norm_keys": [k for k in norm_keys if k in entries],
    }


def upload_artifact(artifact, device):
    """Codebooks to fp32 and every entry tensor to the device
    (infer_compressed_layerwise_triton.py:424-432)."""
    gpu_codebooks = {k: v.to(device, dtype=torch.float32) for k, v in artifact["shared_codebooks"].items()}
    gpu_entries = {k: {ek: (ev.to(device) if torch.is_tensor(ev) else ev) for ek, ev in v.items()}
                   for k, v in artifact["entries"].items()}
    return gpu_codebooks, gpu_entries


def materialize_always_hot(model, plan, gpu_codebooks, device, runtime_dtype):
    """Embedding, lm_head, final norm and rotary buffers on the device
    (infer_compressed_layerwise_triton.py:439-461).  Returns (embed, lm_head)."""
    embed = decode_to_tensor(plan["entries"][plan["embed_key"]], gpu_codebooks, device, runtime_dtype)
    lm_head = embed if plan["lm_head_key"] is None else decode_to_tensor(
        plan["entries"][plan["lm_head_key"]], gpu_codebooks, device, runtime_dtype)
    for key in plan["norm_keys"]:
        val = decode_to_tensor(plan["entries"][key], gpu_codebooks, device, runtime_dtype)
        module = model
        parts = key.split(".")
        for part in parts[:-1]:
            module = getattr(module, part)
        module._parameters[parts[-1]] = torch.nn.Parameter(val, requires_grad=False)
    base = plan["base_model"]
    if hasattr(base, "rotary_emb"):
        base.rotary_emb.to(device)
    return embed, lm_head


def new_kv_cache(base_model):
    """An empty HF key/value cache for the decoder layers."""
    from transformers.cache_utils import DynamicCache
    return DynamicCache(config=base_model.config)


def slots_for(plan, gpu_codebooks, device, runtime_dtype) -> PingPongSlots:
    """The persistent slot manager of this plan (built on first use)."""
    slots = plan.get(_SLOTS_KEY)
    if slots is None or slots.runtime_dtype != runtime_dtype or slots.device != torch.device(device):
        slots = PingPongSlots(plan, gpu_codebooks, device, runtime_dtype)
        plan[_SLOTS_KEY] = slots
    return slots


# ---------------------------------------------------------------------------
# the drop-in forward
# ---------------------------------------------------------------------------

def _layerwise_logits(
    model,
    plan,
    gpu_codebooks,
    embed_weight,
    lm_head_weight,
    input_ids,
    attention_mask,
    past_key_values,
    cache_position,
    device,
    runtime_dtype,
):
    """Reference: infer_compressed_layerwise_triton.py:202-298."""
    base_model = plan["base_model"]
    hidden_states = F.embedding(input_ids, embed_weight)
    position_ids = cache_position.unsqueeze(0)

    position_embeddings = None
    if hasattr(base_model, "rotary_emb"):
        position_embeddings = base_model.rotary_emb(hidden_states, position_ids)

    # same mask choice as the reference (lines 223-238)
    mask_kwargs = {
        "attention_mask": attention_mask,
        "cache_position": cache_position,
        "position_ids": position_ids,
        "past_key_values": past_key_values,
    }
    if hasattr(base_model.forward, "__globals__") and "create_causal_mask" in base_model.forward.__globals__:
        attn_mask = base_model.forward.__globals__["create_causal_mask"](input_embeds=hidden_states, **mask_kwargs)
    else:
        attn_mask = attention_mask

    slots = slots_for(plan, gpu_codebooks, device, runtime_dtype)
    main = torch.cuda.current_stream(device)
    slots.prefetch(0)
    num_layers = len(base_model.layers)
    for layer_idx, layer in enumerate(base_model.layers):
        weights = slots.acquire(layer_idx, main)
        slots.prefetch(layer_idx + 1)
        layer_kwargs = {
            "hidden_states": hidden_states,
            "attention_mask": attn_mask,
            "position_ids": position_ids,
            "past_key_values": past_key_values,
            "use_cache": True,
            "cache_position": cache_position,
        }
        if position_embeddings is not None:
            layer_kwargs["position_embeddings"] = position_embeddings
        with nvtx_range(f"layer_{layer_idx:03d}_forward"):
            hidden_states = functional_call(layer, weights, (), layer_kwargs, strict=False)
        if isinstance(hidden_states, tuple):
            hidden_states = hidden_states[0]
        slots.release(layer_idx, main)
    # the next call starts with layer 0: decode it while the head runs
    slots.prefetch(0)

    hidden_states = base_model.norm(hidden_states)
    logits = F.linear(hidden_states[:, -1:, :], lm_head_weight)
    return logits[:, -1, :], past_key_values


def generate_greedy_ids(model, plan, gpu_codebooks, embed_weight, lm_head_weight, input_ids,
                        max_new_tokens: int, device, runtime_dtype, eos_token_id: Optional[int] = None,
                        forward=None):
    """The token loop of generate_greedy (infer_compressed_layerwise_triton.py:323-386)
    on token ids (no tokenizer).  ``forward`` defaults to this module's
    ``_layerwise_logits`` and may be any function with its signature."""
    forward = forward or _layerwise_logits
    generated = input_ids
    attention = torch.ones_like(input_ids)
    cache = new_kv_cache(plan["base_model"])
    with torch.inference_mode():
        cache_position = torch.arange(generated.shape[1], device=device)
        logits, cache = forward(model, plan, gpu_codebooks, embed_weight, lm_head_weight, generated,
                                attention, cache, cache_position, device, runtime_dtype)
        cache.has_previous_state = True
        all_logits = [logits]
        for _ in range(max_new_tokens):
            next_token = logits.argmax(dim=-1, keepdim=True)
            generated = torch.cat([generated, next_token], dim=1)
            attention = torch.cat([attention, torch.ones_like(next_token)], dim=1)
            if eos_token_id is not None and (next_token == eos_token_id).all():
                break
            cache_position = torch.tensor([generated.shape[1] - 1], device=device)
            logits, cache = forward(model, plan, gpu_codebooks, embed_weight, lm_head_weight,
                                    next_token, attention, cache, cache_position, device, runtime_dtype)
            all_logits.append(logits)
    return generated[:, input_ids.shape[1]:], all_logits
