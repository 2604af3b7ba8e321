"""Qwen3-Next hybrid MoE (80B-A3B architecture): gated DeltaNet + gated attention layers.

The Trainium plugin has no such model; the semantics are those of the public model
definition (HF ``transformers`` ``modeling_qwen3_next.py``):
* layers follow ``layer_types``: three ``linear_attention`` (gated DeltaNet) layers per
  ``full_attention`` layer;
* gated DeltaNet: one projection gives q, k (16 heads x 128), v, z (32 heads x 128), b, a
  (32); a depthwise causal conv (kernel 4) + SiLU over q|k|v; L2-normalised q, k; decay
  g = -exp(A_log) softplus(a + dt_bias), strength beta = sigmoid(b); the gated delta rule;
  a per-head RMSNorm gated by silu(z); out_proj;
* gated attention: q_proj yields (query, gate) per head; QK-norm; partial RoPE (a quarter
  of head_dim 256); output multiplied by sigmoid(gate) before o_proj;
* MoE: softmax router over 512 experts, top-10 renormalised, SiLU-gated experts, plus one
  shared expert scaled by sigmoid(shared_expert_gate(x));
* every RMSNorm except the DeltaNet output norm uses (1 + weight) (stored here as 1 + w).

B200 serving design:
* TP shards attention heads, DeltaNet key heads (with their value heads), the shared
  expert and dense MLP intermediates; routed experts are EP-sharded over the same group;
  each layer returns a partial sum reduced by one fused all-reduce + residual + RMSNorm;
* DeltaNet layers keep per-request state in slots (conv state [slots, C, 3] and recurrent
  state [slots, Hv, 128, 128] fp32) instead of paged KV; prefill runs the chunked state scan,
  decode the recurrent update (``ops.gated_delta_net``);
* our projection row order is [q | k | v | z | b | a] (HF groups rows per key head), so the
  conv input is a prefix of the projection output.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Iterable

import torch
import torch.nn as nn

from .. import ops
from ..nn.linear import ParallelLMHead, RMSNorm, VocabParallelEmbedding, shard_range
from ..ops import reference as ref
from ..parallel.state import GroupCoordinator, ParallelState
from .base import KVSpec, LayerSpec, component, kv_head_sharding
from .llama import DenseMLP, Linear


@dataclass
class Qwen3NextConfig:
    vocab_size: int = 151936
    hidden_size: int = 2048
    num_hidden_layers: int = 48
    num_attention_heads: int = 16
    num_key_value_heads: int = 2
    head_dim: int = 256
    intermediate_size: int = 5120
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10000000.0
    partial_rotary_factor: float = 0.25
    max_position_embeddings: int = 262144
    tie_word_embeddings: bool = False
    linear_conv_kernel_dim: int = 4
    linear_key_head_dim: int = 128
    linear_value_head_dim: int = 128
    linear_num_key_heads: int = 16
    linear_num_value_heads: int = 32
    num_experts: int = 512
    num_experts_per_tok: int = 10
    moe_intermediate_size: int = 512
    shared_expert_intermediate_size: int = 512
    norm_topk_prob: bool = True
    decoder_sparse_step: int = 1
    mlp_only_layers: list = field(default_factory=list)
    layer_types: list | None = None
    quantization: str = "bf16"  # bf16 | fp8 (block-scaled 128x128 checkpoints, dequantised at load)
    mlp_bias: bool = False
    eos_token_id: int | list | None = None

    @classmethod
    def from_hf(cls, d: dict, quantization: str | None = None) -> "Qwen3NextConfig":
        rope = d.get("rope_parameters") or d.get("rope_scaling") or {}
        theta = d.get("rope_theta") or rope.get("rope_theta", 10000000.0)
        prf = d.get("partial_rotary_factor") or rope.get("partial_rotary_factor", 0.25)
        n = d["num_hidden_layers"]
        lt = d.get("layer_types")
        if lt is None:
            iv = d.get("full_attention_interval", 4)
            lt = ["linear_attention" if (i + 1) % iv else "full_attention" for i in range(n)]
        q = quantization
        if q is None:
            qc = d.get("quantization_config") or {}
            q = "fp8" if qc.get("quant_method") == "fp8" else "bf16"
        return cls(vocab_size=d["vocab_size"], hidden_size=d["hidden_size"], num_hidden_layers=n,
                   num_attention_heads=d["num_attention_heads"], num_key_value_heads=d["num_key_value_heads"],
                   head_dim=d.get("head_dim", 256), intermediate_size=d.get("intermediate_size", 5120),
                   rms_norm_eps=d.get("rms_norm_eps", 1e-6), rope_theta=theta, partial_rotary_factor=prf,
                   max_position_embeddings=d.get("max_position_embeddings", 262144),
                   tie_word_embeddings=d.get("tie_word_embeddings", False),
                   linear_conv_kernel_dim=d.get("linear_conv_kernel_dim", 4),
                   linear_key_head_dim=d.get("linear_key_head_dim", 128),
                   linear_value_head_dim=d.get("linear_value_head_dim", 128),
                   linear_num_key_heads=d.get("linear_num_key_heads", 16),
                   linear_num_value_heads=d.get("linear_num_value_heads", 32),
                   num_experts=d.get("num_experts", 512), num_experts_per_tok=d.get("num_experts_per_tok", 10),
                   moe_intermediate_size=d.get("moe_intermediate_size", 512),
                   shared_expert_intermediate_size=d.get("shared_expert_intermediate_size", 512),
                   norm_topk_prob=d.get("norm_topk_prob", True), decoder_sparse_step=d.get("decoder_sparse_step", 1),
                   mlp_only_layers=list(d.get("mlp_only_layers") or []), layer_types=lt, quantization=q,
                   eos_token_id=d.get("eos_token_id"))

    @property
    def rotary_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary_factor)

    def is_moe_layer(self, i: int) -> bool:
        return i not in self.mlp_only_layers and self.num_experts > 0 and (i + 1) % self.decoder_sparse_step == 0


def _param(shape, dtype, device) -> nn.Parameter:
    return nn.Parameter(torch.empty(shape, dtype=dtype, device=device), requires_grad=False)


def dequant_block_fp8(w: torch.Tensor, scale_inv: torch.Tensor, block: int = 128) -> torch.Tensor:
    """Block-scaled fp8 weight [N, K] with fp32 scales [ceil(N/128), ceil(K/128)] -> fp32."""
    N, K = w.shape
    s = scale_inv.float().repeat_interleave(block, 0)[:N].repeat_interleave(block, 1)[:, :K]
    return w.float() * s


class GatedAttention(nn.Module):
    """Full-attention layer with an output gate (see module docstring)."""

    def __init__(self, cfg: Qwen3NextConfig, tp: GroupCoordinator, dtype, device):
        super().__init__()
        t, r = tp.world_size, tp.rank_in_group
        self.tp = tp
        self.nq = cfg.num_attention_heads // t
        self.kv_start, self.nkv = kv_head_sharding(cfg.num_key_value_heads, t, r)
        self.d = cfg.head_dim
        self.rd = cfg.rotary_dim
        self.scale = 1.0 / math.sqrt(self.d)
        self.eps = cfg.rms_norm_eps
        # rows: [q | k | v | gate]
        self.proj = Linear((2 * self.nq + 2 * self.nkv) * self.d, cfg.hidden_size, False, dtype, device)
        self.o_proj = Linear(cfg.hidden_size, self.nq * self.d, False, dtype, device)
        self.q_norm = _param((self.d,), torch.float32, device)
        self.k_norm = _param((self.d,), torch.float32, device)
        self.k_scale = self.v_scale = 1.0

    def load(self, which: str, full: torch.Tensor) -> None:
        d, r, nq = self.d, self.tp.rank_in_group, self.nq
        W = self.proj.weight
        if which == "q":  # HF rows per head: [query(d), gate(d)]
            per = full.view(-1, 2 * d, full.shape[-1])[r * nq:(r + 1) * nq]
            W.data[:nq * d].copy_(per[:, :d].reshape(nq * d, -1).to(W.dtype))
            off = (nq + 2 * self.nkv) * d
            W.data[off:off + nq * d].copy_(per[:, d:].reshape(nq * d, -1).to(W.dtype))
        else:
            rows = full[self.kv_start * d:(self.kv_start + self.nkv) * d]
            off = nq * d if which == "k" else (nq + self.nkv) * d
            W.data[off:off + self.nkv * d].copy_(rows.to(W.dtype))

    def forward(self, positions, x, meta, kv, cos_sin) -> torch.Tensor:
        y = self.proj(x)
        nq, nkv, d = self.nq, self.nkv, self.d
        k_cache, v_cache = kv
        q = ops.rope_and_cache(y, positions, cos_sin, k_cache, v_cache, meta.slot_mapping, nq, nkv, d,
                               self.k_scale, self.v_scale, self.q_norm, self.k_norm, self.eps, self.rd)
        o = ops.attention(q, k_cache, v_cache, meta, self.scale, None, None, self.k_scale, self.v_scale)
        gate = y[:, (nq + 2 * nkv) * d:]
        o = ops.sigmoid_gate_mul(o.reshape(o.shape[0], nq * d), gate)
        return self.o_proj(o)  # partial sum


class GatedDeltaNet(nn.Module):
    """Linear-attention layer (see module docstring); state lives in per-request slots."""

    def __init__(self, cfg: Qwen3NextConfig, tp: GroupCoordinator, dtype, device):
        super().__init__()
        t, r = tp.world_size, tp.rank_in_group
        if cfg.linear_num_key_heads % t:
            raise ValueError(f"linear key heads {cfg.linear_num_key_heads} not divisible by tp {t}")
        self.tp = tp
        self.nk = cfg.linear_num_key_heads // t
        self.rep = cfg.linear_num_value_heads // cfg.linear_num_key_heads
        self.nv = self.nk * self.rep
        self.kh0, self.vh0 = r * self.nk, r * self.nv
        self.dk, self.dv = cfg.linear_key_head_dim, cfg.linear_value_head_dim
        self.K = cfg.linear_conv_kernel_dim
        self.key_dim, self.value_dim = self.nk * self.dk, self.nv * self.dv
        self.conv_dim = 2 * self.key_dim + self.value_dim
        self.eps = cfg.rms_norm_eps
        out = self.conv_dim + self.value_dim + 2 * self.nv
        self.in_proj = Linear(out, cfg.hidden_size, False, dtype, device)
        self.conv_w = _param((self.conv_dim, self.K), dtype, device)
        self.A_log = _param((self.nv,), torch.float32, device)
        self.dt_bias = _param((self.nv,), torch.float32, device)
        self.norm_w = _param((self.dv,), torch.float32, device)
        self.out_proj = Linear(cfg.hidden_size, self.value_dim, False, dtype, device)
        self._full_key_dim = cfg.linear_num_key_heads * self.dk

    def state_shapes(self) -> tuple[tuple[int, int], tuple[int, int, int]]:
        return (self.conv_dim, self.K - 1), (self.nv, self.dk, self.dv)

    def load(self, which: str, full: torch.Tensor) -> None:
        dk, dv, rep, nk, nv = self.dk, self.dv, self.rep, self.nk, self.nv
        W = self.in_proj.weight
        if which == "in_proj_qkvz":
            g = full.view(-1, 2 * dk + 2 * rep * dv, full.shape[-1])[self.kh0:self.kh0 + nk]
            parts = [g[:, :dk], g[:, dk:2 * dk], g[:, 2 * dk:2 * dk + rep * dv], g[:, 2 * dk + rep * dv:]]
            off = 0
            for p in parts:
                p = p.reshape(-1, full.shape[-1])
                W.data[off:off + p.shape[0]].copy_(p.to(W.dtype))
                off += p.shape[0]
        elif which == "in_proj_ba":
            g = full.view(-1, 2 * rep, full.shape[-1])[self.kh0:self.kh0 + nk]
            off = self.conv_dim + self.value_dim
            W.data[off:off + nv].copy_(g[:, :rep].reshape(nv, -1).to(W.dtype))
            W.data[off + nv:off + 2 * nv].copy_(g[:, rep:].reshape(nv, -1).to(W.dtype))
        elif which == "conv1d":
            w = full.reshape(full.shape[0], -1)
            fk = self._full_key_dim
            q = w[self.kh0 * dk:(self.kh0 + nk) * dk]
            k = w[fk + self.kh0 * dk:fk + (self.kh0 + nk) * dk]
            v = w[2 * fk + self.vh0 * dv:2 * fk + (self.vh0 + nv) * dv]
            self.conv_w.data.copy_(torch.cat([q, k, v]).to(self.conv_w.dtype))
        elif which in ("A_log", "dt_bias"):
            getattr(self, which).data.copy_(full[self.vh0:self.vh0 + nv].float())
        elif which == "norm":
            self.norm_w.data.copy_(full.float())
        elif which == "out_proj":
            self.out_proj.weight.data.copy_(full[:, self.vh0 * dv:(self.vh0 + nv) * dv].to(self.out_proj.weight.dtype))
        else:
            raise KeyError(which)

    def forward(self, x, meta, state) -> torch.Tensor:
        conv_state, ssm_state = state
        y = self.in_proj(x)
        cd, vd, nv = self.conv_dim, self.value_dim, self.nv
        mixed = ops.causal_conv1d(y[:, :cd], self.conv_w, conv_state, meta)
        z = y[:, cd:cd + vd]
        b = y[:, cd + vd:cd + vd + nv]
        a = y[:, cd + vd + nv:]
        o = ops.gated_delta_net(mixed, z, b, a, self.A_log, self.dt_bias, self.norm_w, self.eps, ssm_state, meta,
                                self.nk, self.nv, self.dk, self.dv)
        return self.out_proj(o)  # partial sum


class SparseMoE(nn.Module):
    """Routed experts (EP over the group) + TP-sharded shared expert; returns a partial sum."""

    def __init__(self, cfg: Qwen3NextConfig, ps: ParallelState, dtype, device):
        super().__init__()
        self.cfg = cfg
        group = ps.tp
        self.group = group
        self.dp = ps.dp
        E, w = cfg.num_experts, group.world_size * ps.dp.world_size  # EP over TP x DP
        if E % w:
            raise ValueError(f"experts {E} not divisible by the expert-parallel size {w}")
        self.E_local = E // w
        self.e0 = (ps.dp.rank_in_group * group.world_size + group.rank_in_group) * self.E_local
        H, I = cfg.hidden_size, cfg.moe_intermediate_size
        self.router = _param((E, H), dtype, device)
        self.w13 = _param((self.E_local, 2 * I, H), dtype, device)  # [gate | up] rows
        self.w2 = _param((self.E_local, H, I), dtype, device)
        self.shared = DenseMLP(_SharedCfg(H, cfg.shared_expert_intermediate_size), group, dtype, device) \
            if cfg.shared_expert_intermediate_size else None
        self.shared_gate = _param((1, H), dtype, device) if self.shared is not None else None
        self.mx = None  # MXFP8 kernel tensors (set after loading on a GPU for fp8 checkpoints)
        # EP all-to-all (``parallel/all2all.py``), attached by the worker when
        # ``all2all_backend`` asks for one; None: all-gather / reduce-scatter over DP
        self.a2a = None

    def _route(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        k = self.cfg.num_experts_per_tok
        if self.cfg.norm_topk_prob:
            # softmax -> top-k -> renormalise == softmax over the top-k logits
            return ops.router_topk(x, self.router, None, k)
        return ops.router_topk(x, self.router, None, k, "softmax_topk_unnormalized")

    def _experts(self, x: torch.Tensor, ids: torch.Tensor, wts: torch.Tensor) -> torch.Tensor:
        H, I = self.cfg.hidden_size, self.cfg.moe_intermediate_size
        if self.mx is not None:  # MXFP8 experts (fp8 checkpoints on the GPU)
            t13, s13, t2, s2, b13, b2 = self.mx
            return ops.moe_mxfp4(x, ids, wts, t13, s13, b13, t2, s2, b2, self.e0, 1.0, -1.0, H, I, fp4=False)
        return ops.moe_dense(x, ids, wts, self.w13, None, self.w2, None, self.e0, 1.0, None, False, "silu", H, I)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.a2a is not None:
            # each TP rank sends its slice of the local tokens to the expert owners; zeros
            # outside the slice keep the output a TP partial sum
            from ..parallel.all2all import ep_slice

            T = x.shape[0]
            ids, wts = self._route(x)
            t0, t1 = ep_slice(T, self.group.rank_in_group, self.group.world_size)
            xr, ir, wr = self.a2a.dispatch(x, ids, wts, self.E_local, t0, t1)
            out = self.a2a.combine(self._experts(xr, ir, wr), T)
        else:
            xr = self.dp.all_gather(x, dim=0) if self.dp.world_size > 1 else x  # cross-DP expert parallelism
            ids, wts = self._route(xr)
            out = self._experts(xr, ids, wts)
            if self.dp.world_size > 1:
                out = self.dp.reduce_scatter(out, dim=0)
        if self.shared is not None:
            sg = ops.linear(x, self.shared_gate)
            out = ops.gated_add(out, self.shared(x), sg)
        return out

    @torch.no_grad()
    def process_weights_after_loading(self) -> None:
        """On a GPU: re-lay the experts into the grouped-GEMM tiles (gate/up interleaved); fp8
        checkpoints become MXFP8 (e4m3 + ue8m0 per 32), bf16 ones stay bf16."""
        if not (self.w13.is_cuda and self.w13.dim() == 3):
            return
        if self.cfg.quantization == "fp8":
            t13, s13, t2, s2 = ops.prepare_moe_mxfp8(self.w13.data, self.w2.data, interleaved=False)
            dev = t13.device
            z13 = torch.zeros(self.E_local, 2 * self.cfg.moe_intermediate_size, dtype=torch.float32, device=dev)
            z2 = torch.zeros(self.E_local, self.cfg.hidden_size, dtype=torch.float32, device=dev)
            self.mx = (t13, s13, t2, s2, z13, z2)
            self.w13 = nn.Parameter(torch.empty(0, device=dev), requires_grad=False)
            self.w2 = nn.Parameter(torch.empty(0, device=dev), requires_grad=False)
        else:
            t13, t2 = ops.prepare_moe_bf16(self.w13.data, self.w2.data, interleaved=False)
            self.w13 = nn.Parameter(t13, requires_grad=False)
            self.w2 = nn.Parameter(t2, requires_grad=False)


@dataclass
class _SharedCfg:
    hidden_size: int
    intermediate_size: int
    mlp_bias: bool = False
    quantization: str = "bf16"


class Qwen3NextDecoderLayer(nn.Module):
    def __init__(self, cfg: Qwen3NextConfig, i: int, ps: ParallelState, dtype, device):
        super().__init__()
        self.kind = cfg.layer_types[i]
        self.eps = cfg.rms_norm_eps
        self.tp = ps.tp
        self.input_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps, device=device)
        self.post_attention_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps, device=device)
        if self.kind == "linear_attention":
            self.linear_attn = GatedDeltaNet(cfg, ps.tp, dtype, device)
        else:
            self.self_attn = GatedAttention(cfg, ps.tp, dtype, device)
        self.mlp = (SparseMoE(cfg, ps, dtype, device) if cfg.is_moe_layer(i)
                    else DenseMLP(_SharedCfg(cfg.hidden_size, cfg.intermediate_size), ps.tp, dtype, device))

    def forward(self, positions, h, residual, meta, cache, cos_sin):
        if residual is None:
            residual = h
            x = self.input_layernorm(h)
        else:
            x, residual = self.tp.all_reduce_add_rmsnorm(h, residual, self.input_layernorm.weight, self.eps)
        if self.kind == "linear_attention":
            a = self.linear_attn(x, meta, cache)
        else:
            a = self.self_attn(positions, x, meta, cache, cos_sin)
        x, residual = self.tp.all_reduce_add_rmsnorm(a, residual, self.post_attention_layernorm.weight, self.eps)
        return self.mlp(x), residual


class Qwen3NextForCausalLM(nn.Module):
    config_class = Qwen3NextConfig

    def __init__(self, cfg: Qwen3NextConfig, ps: ParallelState, dtype=torch.bfloat16, device="cpu",
                 kv_dtype: torch.dtype | None = None):
        super().__init__()
        self.cfg = cfg
        self.ps = ps
        self.dtype = dtype
        self.kv_dtype = kv_dtype or dtype
        self.embed_tokens = VocabParallelEmbedding(cfg.vocab_size, cfg.hidden_size, dtype=dtype, device=device,
                                                   **component(ps, "embedding"))
        self.layers = nn.ModuleList([Qwen3NextDecoderLayer(cfg, i, ps, dtype, device)
                                     for i in range(cfg.num_hidden_layers)])
        self.norm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps, device=device)
        self.lm_head = ParallelLMHead(cfg.vocab_size, cfg.hidden_size, dtype=dtype, device=device,
                                      **component(ps, "lm_head"))
        inv, af = ref.yarn_inv_freq(cfg.rotary_dim, cfg.rope_theta)
        self.register_buffer("cos_sin", ops.build_cos_sin_cache(inv, min(cfg.max_position_embeddings, 1 << 17), af,
                                                                device=device), persistent=False)
        self.aux_hidden_layers: tuple[int, ...] = ()
        self._aux = None

    # -------------------------------------------------------------- caches
    def get_kv_spec(self) -> KVSpec:
        out = []
        for l in self.layers:
            if l.kind == "linear_attention":
                out.append(LayerSpec(0, 0, self.kv_dtype, None, "linear_attention"))
            else:
                out.append(LayerSpec(l.self_attn.nkv, self.cfg.head_dim, self.kv_dtype))
        return KVSpec(out)

    def get_state_spec(self) -> list:
        """Per layer: None (attention) or ((conv_channels, K-1), (Hv_local, dk, dv))."""
        return [l.linear_attn.state_shapes() if l.kind == "linear_attention" else None for l in self.layers]

    def set_kv_scales(self, k_scale: float, v_scale: float) -> None:
        for l in self.layers:
            if l.kind != "linear_attention":
                l.self_attn.k_scale, l.self_attn.v_scale = k_scale, v_scale

    # -------------------------------------------------------------- forward
    def forward(self, input_ids, positions, meta, kv_caches, inputs_embeds=None):
        h = self.embed_tokens(input_ids) if inputs_embeds is None else inputs_embeds
        residual = None
        for i, layer in enumerate(self.layers):
            h, residual = layer(positions, h, residual, meta, kv_caches[i], self.cos_sin)
        h, _ = self.ps.tp.all_reduce_add_rmsnorm(h, residual, self.norm.weight, self.cfg.rms_norm_eps)
        return h

    def compute_logits(self, h: torch.Tensor) -> torch.Tensor:
        return self.lm_head(h)

    # -------------------------------------------------------------- weights
    def load_weights(self, weights: Iterable[tuple[str, torch.Tensor]]) -> set[str]:
        loaded = set()
        pending_scale: dict[str, torch.Tensor] = {}
        pending_w: dict[str, torch.Tensor] = {}
        for name, t in weights:
            # block-fp8 checkpoints: pair "<x>.weight" (fp8) with "<x>.weight_scale_inv"
            if name.endswith(".weight_scale_inv"):
                base = name[: -len("_scale_inv")]
                if base in pending_w:
                    self._load_one(base, dequant_block_fp8(pending_w.pop(base), t))
                    loaded.add(base)
                else:
                    pending_scale[base] = t
                loaded.add(name)
                continue
            if t.dtype == torch.float8_e4m3fn:
                if name in pending_scale:
                    t = dequant_block_fp8(t, pending_scale.pop(name))
                else:
                    pending_w[name] = t
                    continue
            if self._load_one(name, t):
                loaded.add(name)
        if pending_w:
            raise KeyError(f"fp8 weights without weight_scale_inv: {sorted(pending_w)[:4]}")
        return loaded

    def _load_one(self, name: str, t: torch.Tensor) -> bool:
        n = name[len("model."):] if name.startswith("model.") else name
        if n == "embed_tokens.weight":
            self.embed_tokens.weight.weight_loader(self.embed_tokens.weight, t)
            if self.cfg.tie_word_embeddings:
                self.lm_head.weight.weight_loader(self.lm_head.weight, t)
        elif name == "lm_head.weight":
            self.lm_head.weight.weight_loader(self.lm_head.weight, t)
        elif n == "norm.weight":
            self.norm.weight.data.copy_(1.0 + t.float())
        elif n.startswith("layers."):
            p = n.split(".")
            self._load_layer(self.layers[int(p[1])], p[2:], t)
        else:
            return False
        return True

    def _load_layer(self, layer: Qwen3NextDecoderLayer, p: list[str], t: torch.Tensor) -> None:
        if p[0] in ("input_layernorm", "post_attention_layernorm"):
            getattr(layer, p[0]).weight.data.copy_(1.0 + t.float())
        elif p[0] == "linear_attn":
            la = layer.linear_attn
            la.load(p[1], t)
        elif p[0] == "self_attn":
            at = layer.self_attn
            if p[1] in ("q_norm", "k_norm"):
                getattr(at, p[1]).data.copy_(1.0 + t.float())
            elif p[1] in ("q_proj", "k_proj", "v_proj"):
                at.load(p[1][0], t)
            elif p[1] == "o_proj":
                s, e = shard_range(t.shape[1], at.tp.rank_in_group, at.tp.world_size)
                at.o_proj.weight.data.copy_(t[:, s:e].to(at.o_proj.weight.dtype))
            else:
                raise KeyError(".".join(p))
        elif p[0] == "mlp":
            self._load_mlp(layer.mlp, p[1:], t)
        else:
            raise KeyError(".".join(p))

    def _load_mlp(self, mlp, p: list[str], t: torch.Tensor) -> None:
        if isinstance(mlp, DenseMLP):
            mlp.load(p[0].split("_")[0], p[1], t)
            return
        I = self.cfg.moe_intermediate_size
        if p[0] == "gate":
            mlp.router.data.copy_(t.to(mlp.router.dtype))
        elif p[0] == "shared_expert_gate":
            mlp.shared_gate.data.copy_(t.to(mlp.shared_gate.dtype))
        elif p[0] == "shared_expert":
            mlp.shared.load(p[1].split("_")[0], p[2], t)
        elif p[0] == "experts" and p[1] in ("gate_up_proj", "down_proj"):  # fused 3D tensors
            sl = t[mlp.e0:mlp.e0 + mlp.E_local]
            tgt = mlp.w13 if p[1] == "gate_up_proj" else mlp.w2
            tgt.data.copy_(sl.to(tgt.dtype))
        elif p[0] == "experts":  # per-expert checkpoints: experts.<e>.<gate|up|down>_proj.weight
            e = int(p[1]) - mlp.e0
            if not 0 <= e < mlp.E_local:
                return
            if p[2] == "down_proj":
                mlp.w2.data[e].copy_(t.to(mlp.w2.dtype))
            else:
                off = 0 if p[2] == "gate_proj" else I
                mlp.w13.data[e, off:off + I].copy_(t.to(mlp.w13.dtype))
        else:
            raise KeyError(".".join(p))
