"""Oracle restatement of the reference layerwise engine (engine A).

TEST INFRASTRUCTURE ONLY (tests/ and smoke()).  Restates
``_layerwise_logits`` of infer_compressed_layerwise_triton.py:202-298 and the
token loop of its ``generate_greedy`` (323-386) without streams or slots:
every layer's weights are reconstructed by the numpy oracle
(``rvq_oracle.decode_rvq``, i.e. the reference's ``_decode_rvq_into``), cast to
the runtime dtype and handed to the HF decoder layer with ``functional_call``
(lines 279-294), with the same attention-mask choice (lines 223-238).

Pinned against ``tests/golden/engine_tiny.npz``, produced by the reference
engine itself (tests/golden/make_golden_engine.py).
"""

from __future__ import annotations

import contextlib
from typing import Dict

import numpy as np
import torch
import torch.nn.functional as F

from .rvq_oracle import OUT_F32, RVQEntryNP, decode_rvq

try:
    from torch.func import functional_call
except ImportError:  # pragma: no cover
    from torch.nn.utils.stateless import functional_call


@contextlib.contextmanager
def _meta_parameters():
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


def oracle_weight(entry: Dict[str, object], codebooks, runtime_dtype, device) -> torch.Tensor:
    """Decoded weight of one artifact entry (fp32 values, then the runtime cast)."""
    if entry["method"] == "bf16_raw":
        return entry["data"].to(device=device, dtype=torch.bfloat16).view(*entry["shape"]).to(runtime_dtype)
    cb = codebooks[entry["codebook_id"]].float().cpu().numpy()
    numel = int(np.prod(entry["shape"]))
    e = RVQEntryNP(indices=entry["indices"].cpu().numpy(), codebook=cb,
                   scales=entry["scales"].float().cpu().numpy(), tail=entry["tail"].float().cpu().numpy(),
                   d=int(entry["d"]), group_size=int(entry["group_size"]),
                   trimmed_numel=int(entry["trimmed_numel"]), numel=numel)
    # decode in fp32 (exact), cast once: equal to casting inside the decode
    w32 = torch.from_numpy(decode_rvq(e, OUT_F32).reshape(entry["shape"]))
    return w32.to(runtime_dtype).to(device)


class OracleEngine:
    """Synchronous engine-A forward over oracle-decoded weights."""

    def __init__(self, config, artifact, device, runtime_dtype=torch.bfloat16):
        from transformers import AutoModelForCausalLM
        config._attn_implementation = "eager"
        with _meta_parameters():
            self.model = AutoModelForCausalLM.from_config(config).eval()
        self.base = self.model.model
        self.device = torch.device(device)
        self.dtype = runtime_dtype
        cbs = artifact["shared_codebooks"]
        entries = artifact["entries"]
        n_layers = len(self.base.layers)
        self.layer_weights = []
        for l in range(n_layers):
            pre = f"model.layers.{l}."
            self.layer_weights.append({k[len(pre):]: oracle_weight(v, cbs, runtime_dtype, self.device)
                                       for k, v in entries.items() if k.startswith(pre)})
        self.embed = oracle_weight(entries["model.embed_tokens.weight"], cbs, runtime_dtype, self.device)
        self.lm_head = self.embed
        norm = oracle_weight(entries["model.norm.weight"], cbs, runtime_dtype, self.device)
        self.base.norm._parameters["weight"] = torch.nn.Parameter(norm, requires_grad=False)
        self.base.rotary_emb.to(self.device)

    def layerwise_logits(self, input_ids, attention_mask, past_key_values, cache_position):
        base = self.base
        hidden = F.embedding(input_ids, self.embed)
        position_ids = cache_position.unsqueeze(0)
        position_embeddings = base.rotary_emb(hidden, position_ids)
        if hasattr(base.forward, "__globals__") and "create_causal_mask" in base.forward.__globals__:
            attn_mask = base.forward.__globals__["create_causal_mask"](
                input_embeds=hidden, attention_mask=attention_mask, cache_position=cache_position,
                position_ids=position_ids, past_key_values=past_key_values)
        else:
            attn_mask = attention_mask
        for l, layer in enumerate(base.layers):
            kwargs = {"hidden_states": hidden, "attention_mask": attn_mask, "position_ids": position_ids,
                      "past_key_values": past_key_values, "use_cache": True,
                      "cache_position": cache_position, "position_embeddings": position_embeddings}
            hidden = functional_call(layer, self.layer_weights[l], (), kwargs, strict=False)
            if isinstance(hidden, tuple):
                hidden = hidden[0]
        hidden = base.norm(hidden)
        return F.linear(hidden[:, -1:, :], self.lm_head)[:, -1, :], past_key_values

    def generate(self, prompt_ids, max_new_tokens):
        from transformers.cache_utils import DynamicCache
        cache = DynamicCache(config=self.base.config)
        cache.has_previous_state = False
        generated = prompt_ids
        attention = torch.ones_like(prompt_ids)
        steps = []
        with torch.inference_mode():
            logits, cache = self.layerwise_logits(generated, attention, cache,
                                                  torch.arange(generated.shape[1], device=self.device))
            cache.has_previous_state = True
            steps.append(logits)
            for _ in range(max_new_tokens):
                nxt = logits.argmax(dim=-1, keepdim=True)
                generated = torch.cat([generated, nxt], dim=1)
                attention = torch.cat([attention, torch.ones_like(nxt)], dim=1)
                logits, cache = self.layerwise_logits(
                    nxt, attention, cache, torch.tensor([generated.shape[1] - 1], device=self.device))
                steps.append(logits)
        return generated[:, prompt_ids.shape[1]:], steps
