"""Llama 3 (dense) and the shared dense-decoder building blocks.

Architecture as in the Trainium plugin's ``model/llama3/model.py`` (``LlamaAttention`` :205,
``LlamaMLP`` :894, ``LlamaForCausalLM`` :1404) and HF ``LlamaForCausalLM``: GQA attention
with split-half RoPE (optionally Llama-3.1 frequency scaling), SwiGLU MLP, RMSNorm,
optional tied embeddings.  Qwen3 (the text model of Qwen3-VL) adds per-head RMSNorm on
q and k, which :class:`DenseAttention` supports.

TP: fused QKV and gate|up projections are column-parallel, o_proj and down_proj are
row-parallel and return partial sums; every layer boundary is one fused
all-reduce + residual + RMSNorm (``GroupCoordinator.all_reduce_add_rmsnorm``).
Static per-tensor FP8 (ModelOpt, ``model/llama3/quantization.py``) is supported for the
four linear layers of every block.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Iterable

import torch
import torch.nn as nn

from .. import ops
from ..nn.linear import ParallelLMHead, RMSNorm, VocabParallelEmbedding, shard_range
from ..ops import reference as ref
from ..parallel.state import GroupCoordinator, ParallelState
from .base import KVSpec, LayerSpec, component, kv_head_sharding


@dataclass
class LlamaConfig:
    vocab_size: int = 128256
    hidden_size: int = 4096
    num_hidden_layers: int = 32
    num_attention_heads: int = 32
    num_key_value_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 14336
    rms_norm_eps: float = 1e-5
    rope_theta: float = 500000.0
    rope_scaling: dict | None = None
    max_position_embeddings: int = 131072
    tie_word_embeddings: bool = False
    attention_bias: bool = False
    mlp_bias: bool = False
    qk_norm: bool = False
    quantization: str = "bf16"  # bf16 | fp8
    eos_token_id: int | list | None = None

    @classmethod
    def from_hf(cls, d: dict, quantization: str | None = None) -> "LlamaConfig":
        rope = d.get("rope_scaling") or d.get("rope_parameters")
        theta = d.get("rope_theta") or (rope or {}).get("rope_theta", 10000.0)
        q = quantization
        if q is None:
            qc = d.get("quantization_config") or {}
            q = "fp8" if qc.get("quant_method") in ("modelopt", "fp8") else "bf16"
        return cls(vocab_size=d["vocab_size"], hidden_size=d["hidden_size"], num_hidden_layers=d["num_hidden_layers"],
                   num_attention_heads=d["num_attention_heads"],
                   num_key_value_heads=d.get("num_key_value_heads", d["num_attention_heads"]),
                   head_dim=d.get("head_dim") or d["hidden_size"] // d["num_attention_heads"],
                   intermediate_size=d["intermediate_size"], rms_norm_eps=d.get("rms_norm_eps", 1e-5),
                   rope_theta=theta, rope_scaling=rope if rope and rope.get("rope_type", rope.get("type")) not in
                   (None, "default") else None,
                   max_position_embeddings=d.get("max_position_embeddings", 8192),
                   tie_word_embeddings=d.get("tie_word_embeddings", False),
                   attention_bias=d.get("attention_bias", False), mlp_bias=d.get("mlp_bias", False),
                   qk_norm=d.get("model_type", "").startswith("qwen3"), quantization=q,
                   eos_token_id=d.get("eos_token_id"))

    def inv_freq(self) -> tuple[torch.Tensor, float]:
        rs = self.rope_scaling
        if rs and rs.get("rope_type", rs.get("type")) == "llama3":
            return ref.llama3_inv_freq(self.head_dim, self.rope_theta, rs["factor"], rs["low_freq_factor"],
                                       rs["high_freq_factor"], rs["original_max_position_embeddings"]), 1.0
        if rs and rs.get("rope_type", rs.get("type")) == "yarn":
            return ref.yarn_inv_freq(self.head_dim, self.rope_theta, rs["factor"],
                                     rs.get("original_max_position_embeddings", 4096))
        return ref.yarn_inv_freq(self.head_dim, self.rope_theta)


def _param(shape, dtype, device) -> nn.Parameter:
    return nn.Parameter(torch.empty(shape, dtype=dtype, device=device), requires_grad=False)


class Linear(nn.Module):
    """A local (already sharded) linear layer, bf16 or static FP8.  FP8: e4m3 weight, an fp32
    weight scale per output feature (a per-tensor checkpoint scale is broadcast over the rows
    of its segment, so the q / k / v or gate / up parts of a fused weight keep their own
    scales) and one activation scale (the largest of the fused parts', which quantise the same
    input)."""

    def __init__(self, out_f: int, in_f: int, bias: bool, dtype, device, fp8: bool = False):
        super().__init__()
        self.fp8 = fp8
        self.dtype = dtype
        if fp8:
            self.weight = _param((out_f, in_f), torch.float8_e4m3fn, device)
            self.weight_scale = nn.Parameter(torch.ones(out_f, dtype=torch.float32, device=device), requires_grad=False)
            self.input_scale = nn.Parameter(torch.zeros(1, dtype=torch.float32, device=device), requires_grad=False)
            self.register_buffer("alpha", torch.ones(out_f, dtype=torch.float32, device=device), persistent=False)
        else:
            self.weight = _param((out_f, in_f), dtype, device)
        self.bias = _param((out_f,), dtype, device) if bias else None

    def load_scale(self, kind: str, full: torch.Tensor, rows: slice | None = None) -> None:
        """A checkpoint scale for the output rows ``rows`` (all rows when None)."""
        v = full.float().reshape(-1).to(self.weight_scale.device)
        if kind == "input_scale":
            self.input_scale.data.copy_(torch.maximum(self.input_scale.data, v[:1]))
            return
        tgt = self.weight_scale.data if rows is None else self.weight_scale.data[rows]
        tgt.copy_(v[0].expand_as(tgt) if v.numel() == 1 else v[:tgt.numel()])

    def process_weights_after_loading(self) -> None:
        if self.fp8:
            self.alpha.copy_(self.input_scale.float() * self.weight_scale.float())

    def forward(self, x: torch.Tensor, with_bias: bool = True, x_q: torch.Tensor | None = None) -> torch.Tensor:
        b = self.bias if with_bias else None
        if self.fp8:
            return ops.linear_fp8(x, self.weight, self.weight_scale, self.input_scale, b, x_q=x_q, alpha=self.alpha,
                                  out_dtype=self.dtype)
        return ops.linear(x, self.weight, b)


class DenseAttention(nn.Module):
    def __init__(self, cfg: LlamaConfig, layer_idx: int, tp: GroupCoordinator, dtype, device,
                 sliding_window: int | None = None):
        super().__init__()
        t, r = tp.world_size, tp.rank_in_group
        self.tp = tp
        self.nq = cfg.num_attention_heads // t
        self.kv_start, self.nkv = kv_head_sharding(cfg.num_key_value_heads, t, r)
        self.d = cfg.head_dim
        self.window = sliding_window
        self.scale = 1.0 / math.sqrt(self.d)
        fp8 = cfg.quantization == "fp8"
        self.qkv = Linear((self.nq + 2 * self.nkv) * self.d, cfg.hidden_size, cfg.attention_bias, dtype, device, fp8)
        self.o_proj = Linear(cfg.hidden_size, self.nq * self.d, cfg.attention_bias, dtype, device, fp8)
        self.q_norm = _param((self.d,), torch.float32, device) if cfg.qk_norm else None
        self.k_norm = _param((self.d,), torch.float32, device) if cfg.qk_norm else None
        self.eps = cfg.rms_norm_eps
        self.k_scale = 1.0
        self.v_scale = 1.0

    def load_qkv(self, which: str, kind: str, full: torch.Tensor) -> None:
        d, r = self.d, self.tp.rank_in_group
        if kind in ("weight_scale", "input_scale"):
            nq, nkv = self.nq * d, self.nkv * d
            seg = {"q": slice(0, nq), "k": slice(nq, nq + nkv), "v": slice(nq + nkv, nq + 2 * nkv)}[which]
            if kind == "weight_scale" and full.numel() > 1:  # per-channel: this rank's rows
                rows = slice(r * nq, (r + 1) * nq) if which == "q" else slice(self.kv_start * d,
                                                                              (self.kv_start + self.nkv) * d)
                full = full.reshape(-1)[rows]
            self.qkv.load_scale(kind, full, seg)
            return
        if which == "q":
            rows = slice(r * self.nq * d, (r + 1) * self.nq * d)
            dst = slice(0, self.nq * d)
        else:
            rows = slice(self.kv_start * d, (self.kv_start + self.nkv) * d)
            off = self.nq * d if which == "k" else (self.nq + self.nkv) * d
            dst = slice(off, off + self.nkv * d)
        tgt = self.qkv.weight if kind == "weight" else self.qkv.bias
        tgt.data[dst].copy_(full[rows].to(tgt.dtype))

    def forward(self, positions, x, meta, kv, cos_sin, x_q=None) -> torch.Tensor:
        qkv = self.qkv(x, x_q=x_q)
        k_cache, v_cache = kv
        q = ops.rope_and_cache(qkv, positions, cos_sin, k_cache, v_cache, meta.slot_mapping, self.nq, self.nkv,
                               self.d, self.k_scale, self.v_scale, self.q_norm, self.k_norm, self.eps)
        o = ops.attention(q, k_cache, v_cache, meta, self.scale, None, self.window, self.k_scale, self.v_scale)
        return self.o_proj(o.reshape(o.shape[0], self.nq * self.d), with_bias=False)  # partial sum


class DenseMLP(nn.Module):
    """Gate/up column-parallel, down row-parallel; returns the partial sum over ``tp``.  With
    MLP DP (``dp_group``) ``tp`` is a TP x DP supergroup: the rows of the supergroup's DP
    replicas are gathered, run through the supergroup's shards, and reduce-scattered back,
    leaving each replica a partial sum over its own TP group."""

    def __init__(self, cfg: LlamaConfig, tp: GroupCoordinator, dtype, device, intermediate: int | None = None,
                 dp_group: GroupCoordinator | None = None):
        super().__init__()
        I = intermediate or cfg.intermediate_size
        self.tp = tp
        self.dp_group = dp_group
        self.I_local = I // tp.world_size
        fp8 = cfg.quantization == "fp8"
        self.gate_up = Linear(2 * self.I_local, cfg.hidden_size, cfg.mlp_bias, dtype, device, fp8)
        self.down = Linear(cfg.hidden_size, self.I_local, cfg.mlp_bias, dtype, device, fp8)

    def load(self, which: str, kind: str, full: torch.Tensor) -> None:
        if kind in ("weight_scale", "input_scale"):
            if which == "down":
                self.down.load_scale(kind, full)
                return
            seg = slice(0, self.I_local) if which == "gate" else slice(self.I_local, 2 * self.I_local)
            if kind == "weight_scale" and full.numel() > 1:
                s0, e0 = shard_range(full.numel(), self.tp.rank_in_group, self.tp.world_size)
                full = full.reshape(-1)[s0:e0]
            self.gate_up.load_scale(kind, full, seg)
            return
        r, w = self.tp.rank_in_group, self.tp.world_size
        if which == "down":
            if kind == "weight":
                s, e = shard_range(full.shape[1], r, w)
                self.down.weight.data.copy_(full[:, s:e].to(self.down.weight.dtype))
            else:
                self.down.bias.data.copy_(full.to(self.down.bias.dtype))
            return
        s, e = shard_range(full.shape[0], r, w)
        off = 0 if which == "gate" else self.I_local
        tgt = self.gate_up.weight if kind == "weight" else self.gate_up.bias
        tgt.data[off:off + self.I_local].copy_(full[s:e].to(tgt.dtype))

    def forward(self, x: torch.Tensor, x_q: torch.Tensor | None = None) -> torch.Tensor:
        if self.dp_group is not None:
            xa = self.dp_group.all_gather(x, dim=0)
            return self.dp_group.reduce_scatter(self.down(ops.silu_and_mul(self.gate_up(xa)), with_bias=False), dim=0)
        return self.down(ops.silu_and_mul(self.gate_up(x, x_q=x_q)), with_bias=False)  # partial sum


class DenseDecoderLayer(nn.Module):
    def __init__(self, cfg: LlamaConfig, i: int, ps: ParallelState, dtype, device, sliding_window=None):
        super().__init__()
        self.eps = cfg.rms_norm_eps
        self.tp = ps.tp
        self.input_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps, device=device)
        self.self_attn = DenseAttention(cfg, i, ps.tp, dtype, device, sliding_window)
        self.post_attention_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps, device=device)
        mlp_g, mlp_dp = ps.component("mlp")
        self.mlp = DenseMLP(cfg, mlp_g, dtype, device, dp_group=mlp_dp)

    def _fp8_fused(self) -> bool:
        """Static-FP8 layer on one rank: the norms write e4m3 rows for the FP8 GEMMs directly
        (fused RMSNorm + quantisation) instead of bf16 rows that the GEMM call re-reads."""
        qkv, gu = self.self_attn.qkv, self.mlp.gate_up
        return qkv.fp8 and gu.fp8 and self.tp.world_size == 1 and self.mlp.dp_group is None and \
            not getattr(self.tp, "sp_active", False)

    def forward(self, positions, h, residual, meta, kv, cos_sin, in_bias=None):
        """``h``: the embedding (layer 0) or the previous layer's MLP partial sum, whose
        bias ``in_bias`` is added once after the reduction."""
        if self._fp8_fused():
            at, mlp = self.self_attn, self.mlp
            if in_bias is not None:
                h = h + in_bias
            x_q, residual = ops.rms_norm_fp8(h, self.input_layernorm.weight, self.eps, at.qkv.input_scale, residual)
            if residual is None:
                residual = h
            a = at(positions, None, meta, kv, cos_sin, x_q=x_q)
            if at.o_proj.bias is not None:
                a = a + at.o_proj.bias
            x_q, residual = ops.rms_norm_fp8(a, self.post_attention_layernorm.weight, self.eps,
                                             mlp.gate_up.input_scale, residual)
            return mlp(None, x_q=x_q), residual
        if residual is None:
            residual = h
            x = self.input_layernorm(h)
        else:
            x, residual = self.tp.all_reduce_add_rmsnorm(h, residual, self.input_layernorm.weight, self.eps, in_bias)
        a = self.self_attn(positions, x, meta, kv, cos_sin)
        x, residual = self.tp.all_reduce_add_rmsnorm(a, residual, self.post_attention_layernorm.weight, self.eps,
                                                     self.self_attn.o_proj.bias)
        return self.mlp(x), residual


class LlamaForCausalLM(nn.Module):
    config_class = LlamaConfig

    def __init__(self, cfg: LlamaConfig, ps: ParallelState, dtype=torch.bfloat16, device="cpu",
                 kv_dtype: torch.dtype | None = None):
        super().__init__()
        self.cfg = cfg
        self.ps = ps
        self.dtype = dtype
        self.kv_dtype = kv_dtype or dtype
        self.embed_tokens = VocabParallelEmbedding(cfg.vocab_size, cfg.hidden_size, dtype=dtype, device=device,
                                                   **component(ps, "embedding"))
        self.layers = nn.ModuleList([DenseDecoderLayer(cfg, i, ps, dtype, device)
                                     for i in range(cfg.num_hidden_layers)])
        self.norm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps, device=device)
        self.lm_head = ParallelLMHead(cfg.vocab_size, cfg.hidden_size, dtype=dtype, device=device,
                                      **component(ps, "lm_head"))
        inv, af = cfg.inv_freq()
        self.register_buffer("cos_sin", ops.build_cos_sin_cache(inv, min(cfg.max_position_embeddings, 1 << 17), af,
                                                                device=device), persistent=False)
        self.aux_hidden_layers: tuple[int, ...] = ()
        self._aux = None

    def get_kv_spec(self) -> KVSpec:
        return KVSpec([LayerSpec(l.self_attn.nkv, self.cfg.head_dim, self.kv_dtype, l.self_attn.window)
                       for l in self.layers])

    def set_kv_scales(self, k_scale: float, v_scale: float) -> None:
        for l in self.layers:
            l.self_attn.k_scale, l.self_attn.v_scale = k_scale, v_scale

    def get_eagle3_aux_hidden_state_layers(self) -> tuple[int, ...]:
        """Low / middle / high layers whose inputs feed an EAGLE-3 draft model."""
        n = self.cfg.num_hidden_layers
        return (2, n // 2, n - 3) if n >= 8 else (0, n // 2, n - 1)

    def forward(self, input_ids, positions, meta, kv_caches, inputs_embeds=None):
        h = self.embed_tokens(input_ids) if inputs_embeds is None else inputs_embeds
        residual = None
        aux = []
        prev_bias = None
        for i, layer in enumerate(self.layers):
            if i in self.aux_hidden_layers:
                if residual is None:
                    aux.append(h)
                else:  # hidden state entering layer i = reduced partial (+ bias) + residual
                    red = self.ps.tp.all_reduce(h.clone())
                    aux.append(red + residual if prev_bias is None else red + prev_bias + residual)
            h, residual = layer(positions, h, residual, meta, kv_caches[i], self.cos_sin, prev_bias)
            prev_bias = layer.mlp.down.bias
        last = prev_bias
        h, _ = self.ps.tp.all_reduce_add_rmsnorm(h, residual, self.norm.weight, self.cfg.rms_norm_eps, last)
        self._aux = torch.cat(aux, dim=-1) if aux else None
        return h

    def compute_logits(self, h: torch.Tensor) -> torch.Tensor:
        return self.lm_head(h)

    def load_weights(self, weights: Iterable[tuple[str, torch.Tensor]]) -> set[str]:
        loaded = set()
        for name, t in weights:
            n = name[len("model."):] if name.startswith("model.") else name
            if n == "embed_tokens.weight":
                self.embed_tokens.weight.weight_loader(self.embed_tokens.weight, t)
                if self.cfg.tie_word_embeddings:
                    self.lm_head.weight.weight_loader(self.lm_head.weight, t)
            elif name == "lm_head.weight":
                self.lm_head.weight.weight_loader(self.lm_head.weight, t)
            elif n == "norm.weight":
                self.norm.weight.data.copy_(t.float())
            elif n.startswith("layers."):
                parts = n.split(".")
                self.load_layer(self.layers[int(parts[1])], ".".join(parts[2:]), t)
            else:
                continue
            loaded.add(name)
        return loaded

    @staticmethod
    def load_layer(layer: DenseDecoderLayer, rest: str, t: torch.Tensor) -> None:
        at, mlp = layer.self_attn, layer.mlp
        p = rest.split(".")
        if rest in ("input_layernorm.weight", "post_attention_layernorm.weight"):
            getattr(layer, p[0]).weight.data.copy_(t.float())
        elif p[0] == "self_attn" and p[1] in ("q_proj", "k_proj", "v_proj"):
            at.load_qkv(p[1][0], p[2], t)
        elif p[0] == "self_attn" and p[1] == "o_proj":
            if p[2] == "weight":
                s, e = shard_range(t.shape[1], at.tp.rank_in_group, at.tp.world_size)
                at.o_proj.weight.data.copy_(t[:, s:e].to(at.o_proj.weight.dtype))
            elif p[2] == "bias":
                at.o_proj.bias.data.copy_(t.to(at.o_proj.bias.dtype))
            elif p[2] in ("weight_scale", "input_scale"):
                at.o_proj.load_scale(p[2], t)
        elif p[0] == "self_attn" and p[1] in ("q_norm", "k_norm"):
            getattr(at, p[1]).data.copy_(t.float())
        elif p[0] == "mlp" and p[1] in ("gate_proj", "up_proj", "down_proj"):
            mlp.load(p[1].split("_")[0], p[2], t)
        else:
            raise KeyError(f"unexpected dense-decoder weight {rest}")
