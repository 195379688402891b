"""Batch-1 Qwen3 generation on one GPU with RVQ weights, CUDA-graph captured.

The reference generates token by token through HF decoder layers whose
weights are decoded into a slot every layer (infer_compressed_layerwise_
triton.py:202-298 ``_layerwise_logits``, 301-404 ``generate_greedy``).  Driven
through HF modules, a batch-1 step is dozens of small launches per layer, so
the host launch rate -- not the GPU -- sets ms/token.  ``Qwen3Decoder``
computes the same Qwen3 math with a static KV cache and captures one decode
step in a CUDA graph, so ms/token is device time.  Three weight back ends
share every other op:

* ``dense``: bf16 weights resident, cuBLAS -- the uncompressed model;
* ``slot``:  the reference's dataflow -- each layer's RVQ weights decoded into
  one of two slots (``rvq_decode_layer``, one launch per layer) on a side
  stream one layer ahead, cuBLAS on the slot;
* ``fused``: decode steps never materialise a weight: the lookup-table
  GEMV for every projection (q/k/v in one launch, gate/up in one launch);
* ``fused_exact``: the same launches with exact bf16 weights
  (``rvq_gemv_tiles_exact``): each weight is rebuilt bit-identically to the
  slot's bf16 value and multiplied in fp32, so the products are those of the
  reference's ``F.linear`` on the slot and only the fp32 summation order
  differs (the strict-parity mode for greedy token identity).

Prefill (the prompt, T tokens at once) is a dense contraction; the RVQ modes
run it through the slot pipeline, ``dense`` on its resident weights.

Layer math, HF Qwen3 (modeling_qwen3.Qwen3DecoderLayer):
  x = rmsnorm(h); q, k, v = x Wq^T, x Wk^T, x Wv^T; per-head q_norm / k_norm;
  RoPE (theta from the config); GQA attention over the cache (mask: see
  ``Qwen3Decoder._attention``); h += o(.)
  x = rmsnorm(h); h += down(silu(gate(x)) * up(x)); final rmsnorm; tied lm_head.
RMSNorm statistics and softmax run in fp32, everything else in the runtime
dtype (bf16), rounding at the same points as the HF modules.
"""

from __future__ import annotations

import dataclasses
from dataclasses import dataclass
from typing import Dict, List, Optional

import torch
import torch.distributed as dist
import torch.nn.functional as F

from .engine import LayerDecodePlan, decode_to_tensor
from .gemv import GemvPlan, gemv_supported, interleave_codes, tile_codes
from .slots import SlotArena, SlotSpec

PROJ = ("self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
        "self_attn.o_proj.weight", "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight")
NORMS = ("input_layernorm.weight", "post_attention_layernorm.weight", "self_attn.q_norm.weight",
         "self_attn.k_norm.weight")
MODES = ("dense", "slot", "fused", "fused_exact")


@dataclass
class Dims:
    hidden: int
    intermediate: int
    n_heads: int
    n_kv: int
    head_dim: int
    n_layers: int
    vocab: int
    eps: float
    theta: float

    @classmethod
    def from_config(cls, cfg) -> "Dims":
        theta = getattr(cfg, "rope_theta", None)
        rp = getattr(cfg, "rope_parameters", None)
        if isinstance(rp, dict) and rp.get("rope_theta") is not None:
            theta = rp["rope_theta"]
        return cls(cfg.hidden_size, cfg.intermediate_size, cfg.num_attention_heads,
                   cfg.num_key_value_heads, cfg.head_dim, cfg.num_hidden_layers, cfg.vocab_size,
                   float(cfg.rms_norm_eps), float(theta if theta is not None else 1e6))


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """Qwen3RMSNorm: fp32 statistics, normalised value cast back, times the weight."""
    x32 = x.float()
    x32 = x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + eps)
    return w * x32.to(x.dtype)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


class Qwen3Decoder:
    """Greedy batch-1 generation.  ``artifact``: the compressor's artifact
    dict (``shared_codebooks``, ``entries``); ``config``: an HF Qwen3 config;
    ``causal``: False reproduces the reference engine's attention mask (see
    ``_attention``), True the standard causal one.  ``tp_group``: a NCCL
    process group to run tensor-parallel over (one rank per GPU); the
    artifact is the full model, or this rank's shard when
    ``artifact_is_shard`` (rvq_b200/shard.py layout).  ``tp_reduce``: how the
    native step sums the row-parallel outputs over the ranks: "push" (peer
    stores over NVLink into landing buffers, rvq_b200/tp.py) or "nccl"
    (``dist.all_reduce`` captured in the graph); prefill always uses NCCL.
    ``step_impl``: how a decode step runs -- "native" (one launch per
    operation: rvq_step norms and attention, rvq_gemv_tiles GEMVs, replayed
    from a CUDA graph), "persistent" (fused mode on one GPU: the whole step as
    one cooperative launch, rvq_b200/persist.py, bit-identical to "native") or
    "torch" (the PyTorch ops of the prompt path).  ``slot_decode_ctas``: CTA
    budget of the slot mode's side-stream layer decode (None: half the SMs,
    the budget at which it overlaps the main stream best; 0: every SM)."""

    def __init__(self, config, artifact, device, mode: str = "fused", max_len: int = 512,
                 runtime_dtype: torch.dtype = torch.bfloat16, causal: bool = False,
                 step_impl: str = "native", tp_group=None, artifact_is_shard: bool = False,
                 tp_reduce: str = "push", slot_decode_ctas: Optional[int] = None):
        if mode not in MODES:
            raise ValueError(f"mode must be one of {MODES}")
        if step_impl not in ("native", "torch", "persistent"):
            raise ValueError("step_impl is 'native' (rvq_step kernels), 'persistent' or 'torch'")
        native = step_impl in ("native", "persistent")
        if runtime_dtype != torch.bfloat16 and native:
            raise NotImplementedError("the native decode step computes in bf16")
        if mode == "fused_exact" and step_impl != "native":
            raise NotImplementedError("fused_exact runs on the native decode step")
        if step_impl == "persistent" and (mode != "fused" or tp_group is not None):
            raise NotImplementedError("the persistent decode step runs fused mode on one GPU")
        self.step_impl = step_impl
        self.native = native
        self.slot_decode_ctas = slot_decode_ctas
        self.mode = mode
        self.fused = mode in ("fused", "fused_exact")
        self.device = dev = torch.device(device)
        self.dtype = dt = runtime_dtype
        self.dims = d = Dims.from_config(config)
        # tensor parallelism: column-parallel q/k/v/gate/up, row-parallel o/down
        # followed by an all-reduce of their outputs (rvq_b200/shard.py)
        self.tp_group = tp_group
        self.tp = dist.get_world_size(tp_group) if tp_group is not None else 1
        if tp_reduce not in ("push", "nccl"):
            raise ValueError("tp_reduce is 'push' or 'nccl'")
        self.push = self.tp > 1 and tp_reduce == "push" and native
        self.exchange = None
        if self.tp > 1:
            from .shard import shard_artifact, sharded_dims
            rank = dist.get_rank(tp_group)
            nh, nkv, inter = sharded_dims(d.n_heads, d.n_kv, d.intermediate, self.tp)
            if not artifact_is_shard:
                artifact = shard_artifact(artifact, d.n_layers, rank, self.tp)
            self.dims = d = dataclasses.replace(d, n_heads=nh, n_kv=nkv, intermediate=inter)
        self.max_len = max_len
        self.codebooks = {k: v.to(dev, torch.float32) for k, v in artifact["shared_codebooks"].items()}
        self.entries = {k: {ek: (ev.to(dev) if torch.is_tensor(ev) else ev) for ek, ev in e.items()}
                        for k, e in artifact["entries"].items()}
        E = self.entries
        self.embed = decode_to_tensor(E["model.embed_tokens.weight"], self.codebooks, dev, dt)
        self.lm_head = (decode_to_tensor(E["lm_head.weight"], self.codebooks, dev, dt)
                        if "lm_head.weight" in E else self.embed)
        self.final_norm = decode_to_tensor(E["model.norm.weight"], self.codebooks, dev, dt)
        self.layers: List[Dict[str, object]] = []
        for l in range(d.n_layers):
            pre = f"model.layers.{l}."
            L: Dict[str, object] = {n: decode_to_tensor(E[pre + n], self.codebooks, dev, dt) for n in NORMS}
            L["entries"] = {n: E[pre + n] for n in PROJ}
            self.layers.append(L)
        # HF default rotary: inv_freq = theta^(-2i/hd); cos/sin in fp32, then the runtime dtype
        inv = 1.0 / (d.theta ** (torch.arange(0, d.head_dim, 2, dtype=torch.int64, device=dev).float()
                                 / d.head_dim))
        freqs = torch.outer(torch.arange(max_len, device=dev).float(), inv)
        emb = torch.cat((freqs, freqs), dim=-1)
        self.cos, self.sin = emb.cos().to(dt), emb.sin().to(dt)
        self.scaling = d.head_dim ** -0.5
        self.k_cache = torch.zeros(d.n_layers, d.n_kv, max_len, d.head_dim, dtype=dt, device=dev)
        self.v_cache = torch.zeros_like(self.k_cache)
        self.positions = torch.arange(max_len, device=dev)
        self.causal = causal
        self.valid_bias = torch.tensor(0.0 if causal else 1.0, dtype=dt, device=dev)
        self.neg_inf = torch.tensor(float("-inf"), dtype=dt, device=dev)
        self.causal_bias = torch.full((max_len, max_len), float("-inf"), dtype=dt, device=dev).triu(1)
        self._tok = torch.zeros(1, dtype=torch.long, device=dev)
        self._pos = torch.zeros(1, dtype=torch.long, device=dev)
        self._setup_weights()
        self.persist = None
        if native:
            self._build_step_ops()
        if step_impl == "persistent":
            from .persist import PersistentStep
            self.persist = PersistentStep(self)
        self.graph: Optional[torch.cuda.CUDAGraph] = None

    # -- weights -----------------------------------------------------------------
    def _setup_weights(self) -> None:
        d, dev, dt = self.dims, self.device, self.dtype
        if self.mode == "dense":
            for L in self.layers:
                L["w"] = {n: decode_to_tensor(e, self.codebooks, dev, dt) for n, e in L["entries"].items()}
        else:
            specs = [[SlotSpec(n, tuple(int(s) for s in L["entries"][n]["shape"]), dt) for n in PROJ]
                     for L in self.layers]
            self.arena = SlotArena(specs, dev)
            self.side = torch.cuda.Stream(dev)
            # the side-stream decode of the next layer leaves half the SMs to the
            # layer being computed (otherwise its kernels queue behind the decode)
            ctas = self.slot_decode_ctas
            if ctas is None:
                ctas = torch.cuda.get_device_properties(dev).multi_processor_count // 2
            self.decode_plans = [LayerDecodePlan([(n, L["entries"][n]) for n in PROJ], self.codebooks,
                                                 self.arena.views(l), max_ctas=int(ctas))
                                 for l, L in enumerate(self.layers)]
        # batch-1 activations at fixed addresses (bound by the GEMV plans, reused by graph replays)
        z = lambda n: torch.zeros(n, dtype=dt, device=dev)
        self.x_attn, self.x_mlp = z(d.hidden), z(d.hidden)
        self.q, self.k, self.v = z(d.n_heads * d.head_dim), z(d.n_kv * d.head_dim), z(d.n_kv * d.head_dim)
        self.attn_out, self.o = z(d.n_heads * d.head_dim), z(d.hidden)
        self.gate, self.up, self.act, self.down = z(d.intermediate), z(d.intermediate), z(d.intermediate), z(d.hidden)
        if not self.fused:
            return
        for L in self.layers:
            E = L["entries"]
            for n in PROJ:
                if not gemv_supported(E[n]):
                    raise NotImplementedError(f"fused mode needs rvq_gemv-compatible entries ({n})")
            cb = lambda n: self.codebooks[E[n]["codebook_id"]]
            if self.native:                     # rvq_gemv_tiles plans: _build_step_ops
                for n in PROJ:
                    rows, cols = (int(v) for v in E[n]["shape"])
                    E[n]["codes_tiled"] = tile_codes(E[n]["indices"], rows, cols)
                continue
            for n in PROJ:
                E[n]["codes_il"] = interleave_codes(E[n]["indices"])
            L["gemv_qkv"] = GemvPlan([(E[PROJ[0]], cb(PROJ[0]), self.x_attn, self.q),
                                      (E[PROJ[1]], cb(PROJ[1]), self.x_attn, self.k),
                                      (E[PROJ[2]], cb(PROJ[2]), self.x_attn, self.v)])
            L["gemv_o"] = GemvPlan([(E[PROJ[3]], cb(PROJ[3]), self.attn_out, self.o)])
            L["gemv_gu"] = GemvPlan([(E[PROJ[4]], cb(PROJ[4]), self.x_mlp, self.gate),
                                     (E[PROJ[5]], cb(PROJ[5]), self.x_mlp, self.up)])
            L["gemv_d"] = GemvPlan([(E[PROJ[6]], cb(PROJ[6]), self.act, self.down)])

    def _allreduce(self, t: torch.Tensor) -> torch.Tensor:
        """Sum a row-parallel projection's output over the tensor-parallel ranks."""
        if self.tp > 1:
            dist.all_reduce(t, group=self.tp_group)
        return t

    # -- the layer ------------------------------------------------------------------
    def _attention(self, l: int, q, k, v, pos: Optional[torch.Tensor]) -> torch.Tensor:
        """q [T, nh*hd], k/v [T, nkv*hd] -> [T, nh*hd], as HF's eager attention
        (modeling_qwen3.eager_attention_forward) computes it: bf16 scores
        ``(q k^T) * scaling``, plus the additive mask, fp32 softmax cast to
        bf16, times V.  ``pos`` None: a prompt at positions 0..T-1 (the cache
        restarts); else the [1] position of a single new token.

        The mask is the engine's: the reference passes the 2-D all-ones
        ``attention_mask`` to the layers (its create_causal_mask lookup through
        ``base_model.forward.__globals__`` finds nothing once ``forward`` is
        wrapped, as it is in transformers 5.x), which adds 1.0 to every score
        and masks nothing, so prompt tokens attend both ways.  ``causal=True``
        gives the standard causal Qwen3 forward instead."""
        d, L = self.dims, self.layers[l]
        T = q.shape[0]
        rep = d.n_heads // d.n_kv
        q = rmsnorm(q.view(1, T, d.n_heads, d.head_dim), L["self_attn.q_norm.weight"], d.eps).transpose(1, 2)
        k = rmsnorm(k.view(1, T, d.n_kv, d.head_dim), L["self_attn.k_norm.weight"], d.eps).transpose(1, 2)
        v = v.view(1, T, d.n_kv, d.head_dim).transpose(1, 2)
        idx = self.positions[:T] if pos is None else pos
        cos = self.cos.index_select(0, idx).view(1, 1, T, d.head_dim)
        sin = self.sin.index_select(0, idx).view(1, 1, T, d.head_dim)
        q = q * cos + rotate_half(q) * sin                 # [1, nh, T, hd]
        k = k * cos + rotate_half(k) * sin                 # [1, nkv, T, hd]
        kc, vc = self.k_cache[l], self.v_cache[l]
        if pos is None:
            # the prompt: exactly the engine's ops (repeat_kv, batched matmuls)
            kc[:, :T].copy_(k[0])
            vc[:, :T].copy_(v[0])
            kr = k[:, :, None].expand(1, d.n_kv, rep, T, d.head_dim).reshape(1, d.n_heads, T, d.head_dim)
            vr = v[:, :, None].expand(1, d.n_kv, rep, T, d.head_dim).reshape(1, d.n_heads, T, d.head_dim)
            s = torch.matmul(q, kr.transpose(2, 3)) * self.scaling
            if self.causal:
                s = s + self.causal_bias[:T, :T]
            else:
                s = s + 1
            p = torch.softmax(s, dim=-1, dtype=torch.float32).to(q.dtype)
            out = torch.matmul(p, vr)                       # [1, nh, T, hd]
            return out.transpose(1, 2).reshape(T, d.n_heads * d.head_dim)
        # one new token over the static cache; keys past ``pos`` get -inf
        kc.index_copy_(1, pos, k[0])
        vc.index_copy_(1, pos, v[0])
        qg = q.view(d.n_kv, rep, d.head_dim)               # GQA without copying the cache
        s = torch.matmul(qg, kc.transpose(1, 2)) * self.scaling       # [nkv, rep, max_len]
        bias = torch.where(self.positions <= pos, self.valid_bias, self.neg_inf)
        p = torch.softmax(s + bias, dim=-1, dtype=torch.float32).to(q.dtype)
        return torch.matmul(p, vc).view(1, d.n_heads * d.head_dim)

    def _layer(self, l: int, h: torch.Tensor, pos, w, gemv: bool) -> torch.Tensor:
        d, L = self.dims, self.layers[l]
        x = rmsnorm(h, L["input_layernorm.weight"], d.eps)
        if gemv:
            self.x_attn.copy_(x.view(-1))
            L["gemv_qkv"].launch()
            q, k, v = self.q.view(1, -1), self.k.view(1, -1), self.v.view(1, -1)
        else:
            q = F.linear(x, w[PROJ[0]])
            k = F.linear(x, w[PROJ[1]])
            v = F.linear(x, w[PROJ[2]])
        a = self._attention(l, q, k, v, pos)
        if gemv:
            self.attn_out.copy_(a.view(-1))
            L["gemv_o"].launch()
            o = self.o.view(1, -1)
        else:
            o = F.linear(a, w[PROJ[3]])
        h = h + self._allreduce(o)
        x = rmsnorm(h, L["post_attention_layernorm.weight"], d.eps)
        if gemv:
            self.x_mlp.copy_(x.view(-1))
            L["gemv_gu"].launch()
            torch.mul(F.silu(self.gate), self.up, out=self.act)
            L["gemv_d"].launch()
            dn = self.down.view(1, -1)
        else:
            dn = F.linear(F.silu(F.linear(x, w[PROJ[4]])) * F.linear(x, w[PROJ[5]]), w[PROJ[6]])
        return h + self._allreduce(dn)

    def _layer_weights(self, slots: bool):
        """Yield (layer, weights) in order.  With ``slots``, layer l+1 is decoded
        into the other slot on the side stream while layer l computes: the
        main stream waits for ready[l % 2], the side stream for free[(l+1) % 2]
        (recorded after the last reader of that slot)."""
        d = self.dims
        if not slots:
            for l in range(d.n_layers):
                yield l, (self.layers[l]["w"] if self.mode == "dense" else None)
            return
        main = torch.cuda.current_stream(self.device)
        ready = [torch.cuda.Event() for _ in range(2)]
        free = [torch.cuda.Event() for _ in range(2)]
        self.side.wait_stream(main)
        with torch.cuda.stream(self.side):
            self.decode_plans[0].launch()
            ready[0].record(self.side)
        for l in range(d.n_layers):
            main.wait_event(ready[l % 2])
            if l + 1 < d.n_layers:
                with torch.cuda.stream(self.side):
                    if l >= 1:
                        self.side.wait_event(free[(l + 1) % 2])
                    self.decode_plans[l + 1].launch()
                    ready[(l + 1) % 2].record(self.side)
            yield l, self.arena.views(l)
            free[l % 2].record(main)
        main.wait_stream(self.side)

    def _forward(self, ids: torch.Tensor, pos: Optional[torch.Tensor]) -> torch.Tensor:
        """ids [T] -> logits of the last position [vocab] with PyTorch ops
        (the prompt; and decode steps when ``step_impl == "torch"``)."""
        d = self.dims
        h = self.embed.index_select(0, ids)
        gemv = self.fused and pos is not None
        for l, w in self._layer_weights(self.mode != "dense" and not gemv):
            h = self._layer(l, h, pos, w, gemv)
        h = rmsnorm(h[-1:], self.final_norm, d.eps)
        return F.linear(h, self.lm_head).view(-1)

    # -- the native decode step --------------------------------------------------------
    def _build_step_ops(self) -> None:
        """Kernel descriptors of the native decode step (one token at ``self._pos``)."""
        from .step import AttentionOp, NormOp, SiluMulOp
        d, dev, dt = self.dims, self.device, self.dtype
        self.h = torch.zeros(d.hidden, dtype=dt, device=dev)
        self.x_final = torch.zeros(d.hidden, dtype=dt, device=dev)
        self.logits_buf = torch.zeros(d.vocab, dtype=dt, device=dev)
        # tensor parallel: each rank computes the logits of its vocab slice of
        # the (replicated) head, then one all-gather inside the step
        self.head_sharded = self.tp > 1 and d.vocab % self.tp == 0
        if self.head_sharded:
            rank, part = dist.get_rank(self.tp_group), d.vocab // self.tp
            self.lm_head_local = self.lm_head[rank * part:(rank + 1) * part]
            self.logits_local = torch.zeros(part, dtype=dt, device=dev)
        self.step_ops = []
        fused = self.fused
        exact = self.mode == "fused_exact"
        if fused:
            # projection outputs stay as per-tile fp32 partials; consumers add the tiles
            from .gemv import GemvTilesPlan, tiles_count
            part = lambda rows, cols: torch.zeros(tiles_count(cols), rows, dtype=torch.float32, device=dev)
            qd, kvd = d.n_heads * d.head_dim, d.n_kv * d.head_dim
            self.q_part, self.k_part, self.v_part = part(qd, d.hidden), part(kvd, d.hidden), part(kvd, d.hidden)
            self.o_part = part(d.hidden, qd)
            self.gate_part, self.up_part = part(d.intermediate, d.hidden), part(d.intermediate, d.hidden)
            self.down_part = part(d.hidden, d.intermediate)
            q, k, v, o, down = self.q_part, self.k_part, self.v_part, self.o_part, self.down_part
            if self.tp > 1 and not self.push:
                # row-parallel outputs: tiles summed locally, then one fp32 vector all-reduced
                self.o_red = torch.zeros(d.hidden, dtype=torch.float32, device=dev)
                self.down_red = torch.zeros(d.hidden, dtype=torch.float32, device=dev)
                o, down = self.o_red, self.down_red
        else:
            q, k, v, o, down = self.q, self.k, self.v, self.o, self.down
        tiles = lambda t: t.shape[0] if t.dim() == 2 else 1
        land_o = land_d = None
        if self.push:
            # row-parallel outputs pushed to every rank's landing buffer; the norms wait and add
            from .tp import PeerExchange, TpPushOp
            self.exchange = PeerExchange(self.tp_group, d.hidden, dev)
            self.push_o = TpPushOp(self.exchange, "o", o, tiles(o))
            self.push_down = TpPushOp(self.exchange, "down", down, tiles(down))
            land_o, land_d = self.exchange.landing("o"), self.exchange.landing("down")
        for l, L in enumerate(self.layers):
            first = l == 0
            ops = {
                "norm1": NormOp(self.h, L["input_layernorm.weight"], self.x_attn, d.eps,
                                add=None if first or land_d else down, add_tiles=tiles(down),
                                token=self._tok if first else None, embed=self.embed if first else None,
                                landing=None if first else land_d),
                "attn": AttentionOp(q, k, v, L["self_attn.q_norm.weight"],
                                    L["self_attn.k_norm.weight"], self.cos, self.sin, self._pos,
                                    self.k_cache[l], self.v_cache[l], self.attn_out, n_heads=d.n_heads,
                                    n_kv=d.n_kv, head_dim=d.head_dim, eps=d.eps, scaling=self.scaling,
                                    valid_bias=0.0 if self.causal else 1.0, q_tiles=tiles(q), kv_tiles=tiles(k)),
                "norm2": NormOp(self.h, L["post_attention_layernorm.weight"], self.x_mlp, d.eps,
                                add=None if land_o else o, add_tiles=tiles(o), landing=land_o),
            }
            if fused:
                E = L["entries"]
                cb = lambda n: self._cb_tiles(E[n]["codebook_id"])
                ops["qkv"] = GemvTilesPlan([(E[PROJ[0]], cb(PROJ[0]), self.x_attn, self.q_part),
                                            (E[PROJ[1]], cb(PROJ[1]), self.x_attn, self.k_part),
                                            (E[PROJ[2]], cb(PROJ[2]), self.x_attn, self.v_part)], exact=exact)
                ops["o"] = GemvTilesPlan([(E[PROJ[3]], cb(PROJ[3]), self.attn_out, self.o_part)], exact=exact)
                ops["gu"] = GemvTilesPlan([(E[PROJ[4]], cb(PROJ[4]), self.x_mlp, self.gate_part),
                                           (E[PROJ[5]], cb(PROJ[5]), self.x_mlp, self.up_part)], exact=exact)
                ops["down"] = GemvTilesPlan([(E[PROJ[6]], cb(PROJ[6]), self.up_part, self.down_part,
                                              self.gate_part)], exact=exact)      # silu(gate) * up fused in
            else:
                ops["silu"] = SiluMulOp(self.gate, self.up, self.act)
            self.step_ops.append(ops)
        self.final_op = NormOp(self.h, self.final_norm, self.x_final, d.eps, add=None if land_d else down,
                               add_tiles=tiles(down), landing=land_d)

    def _cb_tiles(self, cid: str) -> torch.Tensor:
        """The codebook handed to rvq_gemv_tiles: fp16 when every value is an
        fp16 number (the artifact stores fp16 codebooks; the kernel then loads
        it without converting), else the fp32 copy."""
        cache = self.__dict__.setdefault("_cb16", {})
        if cid not in cache:
            cb = self.codebooks[cid]
            h = cb.to(torch.float16)
            cache[cid] = h if torch.equal(h.to(cb.dtype), cb) else cb
        return cache[cid]

    @staticmethod
    def _mv(w: torch.Tensor, x: torch.Tensor, y: torch.Tensor) -> None:
        torch.mm(x.view(1, -1), w.t(), out=y.view(1, -1))         # = F.linear(x, w)

    def _step_native(self) -> torch.Tensor:
        fused = self.fused
        for l, w in self._layer_weights(self.mode == "slot"):
            ops = self.step_ops[l]
            ops["norm1"].launch()
            if fused:
                ops["qkv"].launch()
            else:
                self._mv(w[PROJ[0]], self.x_attn, self.q)
                self._mv(w[PROJ[1]], self.x_attn, self.k)
                self._mv(w[PROJ[2]], self.x_attn, self.v)
            ops["attn"].launch()
            if fused:
                ops["o"].launch()
            else:
                self._mv(w[PROJ[3]], self.attn_out, self.o)
            if self.push:
                self.push_o.launch()
            elif fused and self.tp > 1:
                torch.sum(self.o_part, 0, out=self.o_red)
                self._allreduce(self.o_red)
            elif not fused:
                self._allreduce(self.o)
            ops["norm2"].launch()
            if fused:
                ops["gu"].launch()
                ops["down"].launch()
            else:
                self._mv(w[PROJ[4]], self.x_mlp, self.gate)
                self._mv(w[PROJ[5]], self.x_mlp, self.up)
                ops["silu"].launch()
                self._mv(w[PROJ[6]], self.act, self.down)
            if self.push:
                self.push_down.launch()
            elif fused and self.tp > 1:
                torch.sum(self.down_part, 0, out=self.down_red)
                self._allreduce(self.down_red)
            elif not fused:
                self._allreduce(self.down)
        self.final_op.launch()
        if self.head_sharded:
            self._mv(self.lm_head_local, self.x_final, self.logits_local)
            dist.all_gather_into_tensor(self.logits_buf, self.logits_local, group=self.tp_group)
        else:
            self._mv(self.lm_head, self.x_final, self.logits_buf)
        return self.logits_buf

    def _step_persistent(self) -> torch.Tensor:
        """The native step as one cooperative launch (rvq_b200/persist.py), then the head."""
        self.persist.launch()
        self._mv(self.lm_head, self.x_final, self.logits_buf)
        return self.logits_buf

    # -- prefill (eager) and graph-replayed decode steps -------------------------------
    def prefill(self, prompt: torch.Tensor) -> torch.Tensor:
        """Prompt ids [T] (device) -> last-position logits; cache rows 0..T-1 written."""
        if prompt.numel() > self.max_len:
            raise ValueError("prompt longer than the cache")
        with torch.inference_mode():
            return self._forward(prompt.view(-1), None)

    def capture(self) -> "Qwen3Decoder":
        """Record one decode step (token ``self._tok`` at ``self._pos``) as a CUDA graph."""
        kv = (self.k_cache.clone(), self.v_cache.clone())
        run = {"native": self._step_native, "persistent": self._step_persistent}.get(
            self.step_impl, lambda: self._forward(self._tok, self._pos))
        with torch.inference_mode():
            s = torch.cuda.Stream(self.device)
            s.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(s):
                for _ in range(2):
                    self._logits = run()
            torch.cuda.current_stream(self.device).wait_stream(s)
            torch.cuda.synchronize(self.device)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self._logits = run()
        self.k_cache.copy_(kv[0])                         # warm-up steps wrote row 0
        self.v_cache.copy_(kv[1])
        return self

    def step(self, token: torch.Tensor, pos: int) -> torch.Tensor:
        """One decode step by graph replay; ``token`` a device tensor of one id."""
        if self.graph is None:
            self.capture()
        if not 0 <= pos < self.max_len:
            raise ValueError("position outside the cache")
        self._tok.copy_(token.view(1))
        self._pos.fill_(pos)
        self.graph.replay()
        return self._logits

    def check_waits(self) -> None:
        """Raise if a bounded device wait of this decoder's kernels gave up
        since the last check: a tensor-parallel landing-buffer wait (the norm
        then summed whatever the buffer held), a fused GEMV's wait for its
        code copies, or a phase wait of the persistent step.  Any of them
        makes the logits of that step invalid.
        Synchronises the device."""
        torch.cuda.synchronize(self.device)
        failed = []
        with torch.cuda.device(self.device):
            if self.push:
                from .tp import take_timeout
                if take_timeout():
                    failed.append("a tensor-parallel landing-buffer wait")
            if self.mode == "fused" and self.step_impl == "native":      # the table GEMV's bulk copies
                from .gemv import take_wait_timeout
                if take_wait_timeout():
                    failed.append("a fused GEMV code-copy wait")
            if self.persist is not None and self.persist.take_error():
                failed.append("a persistent-step phase or code-copy wait")
        if failed:
            raise RuntimeError(" and ".join(failed) + " timed out; the generated tokens are invalid")

    def close(self) -> None:
        """Release the captured graph and, collectively over the tensor-parallel
        group, the peer landing buffers.  Every rank calls it at the same point."""
        self.graph = None
        if self.exchange is not None:
            torch.cuda.synchronize(self.device)
            from .tp import take_timeout
            timed_out = take_timeout()
            self.exchange.close()
            self.exchange = None
            if timed_out:
                raise RuntimeError("a tensor-parallel landing-buffer wait timed out")

    def generate(self, prompt: torch.Tensor, new_tokens: int, return_logits: bool = False):
        """Greedy: prompt ids [T] (device) -> ``new_tokens`` ids (device [new_tokens])."""
        if self.graph is None:
            self.capture()
        logits = self.prefill(prompt)
        toks, all_logits = [], [logits.float().clone()] if return_logits else None
        pos = prompt.numel()
        tok = logits.argmax().view(1)
        for i in range(new_tokens):
            toks.append(tok)
            if i + 1 == new_tokens:
                break
            logits = self.step(tok, pos)
            if return_logits:
                all_logits.append(logits.float().clone())
            pos += 1
            tok = logits.argmax().view(1)
        ids = torch.cat(toks)
        self.check_waits()
        return (ids, all_logits) if return_logits else ids
