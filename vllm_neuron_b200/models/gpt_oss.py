"""GPT-OSS (20B / 120B architecture).

Architecture as in the Trainium plugin's ``model/gpt_oss/model_mxfp4.py`` (and HF
``GptOssForCausalLM``): GQA attention with per-head sink logits (``:360-362``),
sliding window 128 on even layers (``:267``), YaRN RoPE (``:141-197``), a replicated
top-k softmax router with bias (``:949-955``), clamped SwiGLU experts with
interleaved gate/up rows (``:1104,1207-1211``), MXFP4 expert weights from the HF
``*_blocks`` / ``*_scales`` keys (``:2114-2132``).

B200 design:
* H stays 2880 (no padding to 3072): 2880 = 90 MX blocks, kernels tile K by 32/64.
* attention is TP-sharded over the TP group; the fused QKV projection is one GEMM,
  RoPE + paged-KV write is one kernel, attention reads the paged cache.
* experts are EP-sharded: rank r owns experts ``[r*E/ep, (r+1)*E/ep)`` with the full
  intermediate dimension; MXFP4 weights stay packed (the tensor-core operand
  format) and the MoE output is completed by one all-reduce (decode), as in the
  reference's ``moe_block_tkg + all_reduce`` path (``model_mxfp4.py:1329-1330``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Iterable

import torch
import torch.nn as nn

from .. import envs, ops
from ..nn.linear import ParallelLMHead, RMSNorm, RowParallelLinear, VocabParallelEmbedding
from ..ops import reference as ref
from ..ops.mx_layout import round_up, scales_to_atoms, tile_values, tiled_shape
from ..parallel.state import GroupCoordinator, ParallelState, RoutePartial
from .base import KVSpec, LayerSpec, component, kv_head_sharding


@dataclass
class GptOssConfig:
    vocab_size: int = 201088
    hidden_size: int = 2880
    num_hidden_layers: int = 24
    num_attention_heads: int = 64
    num_key_value_heads: int = 8
    head_dim: int = 64
    intermediate_size: int = 2880
    num_local_experts: int = 32
    num_experts_per_tok: int = 4
    sliding_window: int = 128
    layer_types: list | None = None
    rope_theta: float = 150000.0
    rope_scaling: dict | None = None
    rms_norm_eps: float = 1e-5
    swiglu_limit: float = 7.0
    swiglu_alpha: float = 1.702
    attention_bias: bool = True
    max_position_embeddings: int = 131072
    quantization: str = "mxfp4"  # mxfp4 | bf16
    tie_word_embeddings: bool = False
    eos_token_id: int | list | None = None

    @classmethod
    def from_hf(cls, d: dict, quantization: str | None = None) -> "GptOssConfig":
        rope = d.get("rope_scaling") or d.get("rope_parameters")
        theta = d.get("rope_theta") or (rope or {}).get("rope_theta", 150000.0)
        q = quantization
        if q is None:
            qc = d.get("quantization_config") or {}
            q = "mxfp4" if qc.get("quant_method") == "mxfp4" else "bf16"
        n_layers = d["num_hidden_layers"]
        lt = d.get("layer_types") or [
            "sliding_attention" if i % 2 == 0 else "full_attention" for i in range(n_layers)
        ]
        return cls(vocab_size=d["vocab_size"], hidden_size=d["hidden_size"], num_hidden_layers=n_layers,
                   num_attention_heads=d["num_attention_heads"], num_key_value_heads=d["num_key_value_heads"],
                   head_dim=d.get("head_dim") or d["hidden_size"] // d["num_attention_heads"],
                   intermediate_size=d["intermediate_size"], num_local_experts=d["num_local_experts"],
                   num_experts_per_tok=d.get("num_experts_per_tok", d.get("experts_per_token", 4)),
                   sliding_window=d.get("sliding_window", 128), layer_types=lt, rope_theta=theta,
                   rope_scaling=rope if rope and rope.get("rope_type", rope.get("type")) == "yarn" else None,
                   rms_norm_eps=d.get("rms_norm_eps", 1e-5), swiglu_limit=d.get("swiglu_limit", 7.0),
                   attention_bias=d.get("attention_bias", True),
                   max_position_embeddings=d.get("max_position_embeddings", 131072), quantization=q,
                   tie_word_embeddings=d.get("tie_word_embeddings", False), eos_token_id=d.get("eos_token_id"))

    def layer_window(self, i: int) -> int | None:
        lt = self.layer_types or ["sliding_attention" if j % 2 == 0 else "full_attention"
                                  for j in range(self.num_hidden_layers)]
        return self.sliding_window if lt[i] == "sliding_attention" else None

    def rope_params(self) -> tuple[torch.Tensor, float]:
        rs = self.rope_scaling
        if rs:
            return ref.yarn_inv_freq(self.head_dim, self.rope_theta, rs.get("factor", 1.0),
                                     rs.get("original_max_position_embeddings", 4096), rs.get("beta_fast", 32.0),
                                     rs.get("beta_slow", 1.0), rs.get("truncate", False))
        return ref.yarn_inv_freq(self.head_dim, self.rope_theta)


def _param(shape, dtype, device) -> nn.Parameter:
    return nn.Parameter(torch.empty(shape, dtype=dtype, device=device), requires_grad=False)


def _pad_narrow(t: torch.Tensor, dim: int, full: int, padded: int, start: int, length: int) -> torch.Tensor:
    """``t`` (size ``full`` along ``dim``) zero-padded to ``padded``, then [start, start+length)."""
    if t.shape[dim] != full:
        raise ValueError(f"expected {full} entries along dim {dim}, got {t.shape[dim]}")
    if padded > full:
        shape = list(t.shape)
        shape[dim] = padded - full
        t = torch.cat([t, torch.zeros(shape, dtype=t.dtype, device=t.device)], dim)
    return t.narrow(dim, start, length)


def _attention_dp(ps: ParallelState) -> GroupCoordinator | None:
    """The attention-DP group (DP replicas at one TP position) when attention DP is on."""
    g = getattr(ps, "attn_dp", None)
    return g if (g is not None and g.world_size > 1) else None


def _single_group() -> GroupCoordinator:
    from ..parallel.state import _single

    return _single("dp")


class GptOssAttention(nn.Module):
    """GQA with sinks over the paged cache; q heads and the o_proj input columns sharded
    over ``tp``.

    Attention DP (``adp``, ``attention_decode.py:530-563,756-765``, ``model_mxfp4.py:274-339``):
    ``tp`` is then a supergroup of a = adp.world_size DP replicas x TP ranks that holds the
    tokens of all a replicas.  The q projection is sharded over the supergroup, the member at
    TP position t of replica j taking q shard t * a + j, so the a members at position t hold
    together exactly the heads of plain TP rank t; K/V are projected with TP rank t's kv
    heads.  An all-to-all over ``adp`` swaps batch for heads: each rank attends its own
    replica's tokens (own KV cache and metadata) with TP rank t's heads, and the reverse
    all-to-all returns its q shard for every token to the o_proj.  KV heads never move."""

    def __init__(self, cfg: GptOssConfig, layer_idx: int, tp: GroupCoordinator, dtype, device,
                 adp: GroupCoordinator | None = None):
        super().__init__()
        self.cfg = cfg
        self.tp = tp
        self.adp = adp
        self.layer_idx = layer_idx
        t, r = tp.world_size, tp.rank_in_group
        if cfg.num_attention_heads % t:
            raise ValueError("attention heads must divide by tp")
        self.nq = cfg.num_attention_heads // t
        if adp is None:
            self.q_shard = r
            self.kv_start, self.nkv = kv_head_sharding(cfg.num_key_value_heads, t, r)
            self.head0, self.nq_attn = r * self.nq, self.nq
        else:
            a, j = adp.world_size, adp.rank_in_group
            tp_plain = t // a
            tpos = r % tp_plain
            self.q_shard = tpos * a + j
            self.kv_start, self.nkv = kv_head_sharding(cfg.num_key_value_heads, tp_plain, tpos)
            self.nq_attn = cfg.num_attention_heads // tp_plain
            self.head0 = tpos * self.nq_attn
        self.d = cfg.head_dim
        self.window = cfg.layer_window(layer_idx)
        self.scale = 1.0 / math.sqrt(self.d)
        qkv_out = (self.nq + 2 * self.nkv) * self.d
        self.qkv_weight = _param((qkv_out, cfg.hidden_size), dtype, device)
        self.qkv_bias = _param((qkv_out,), dtype, device) if cfg.attention_bias else None
        self.sinks = _param((self.nq_attn,), torch.float32, device)
        self.o_proj = RowParallelLinear(cfg.num_attention_heads * self.d, cfg.hidden_size, tp,
                                        bias=cfg.attention_bias, dtype=dtype, device=device)
        if adp is not None:  # o_proj input columns follow the q shard, not the group rank
            qs, w = self.q_shard, self.nq * self.d
            self.o_proj.weight.weight_loader = lambda p, full: p.data.copy_(full[:, qs * w:(qs + 1) * w].to(p.dtype))
        self.k_scale = 1.0
        self.v_scale = 1.0

    # -- weight loading -------------------------------------------------------
    def load_q_k_v(self, which: str, kind: str, full: torch.Tensor) -> None:
        d, r = self.d, self.q_shard
        if which == "q":
            rows = slice(r * self.nq * d, (r + 1) * self.nq * d)
            dst = slice(0, self.nq * d)
        else:
            rows = slice(self.kv_start * d, (self.kv_start + self.nkv) * d)
            off = self.nq * d if which == "k" else (self.nq + self.nkv) * d
            dst = slice(off, off + self.nkv * d)
        if kind == "weight":
            self.qkv_weight.data[dst].copy_(full[rows].to(self.qkv_weight.dtype))
        else:
            self.qkv_bias.data[dst].copy_(full[rows].to(self.qkv_bias.dtype))

    def load_sinks(self, full: torch.Tensor) -> None:
        self.sinks.data.copy_(full[self.head0:self.head0 + self.nq_attn].float())

    def forward(self, positions: torch.Tensor, x: torch.Tensor, meta, kv: tuple, cos_sin: torch.Tensor
                ) -> torch.Tensor:
        """This rank's partial output projection (reduced by the caller)."""
        o = self.attend(positions, x, meta, kv, cos_sin)
        return ops.linear(o, self.o_proj.weight, None)

    def attend(self, positions: torch.Tensor, x: torch.Tensor, meta, kv: tuple, cos_sin: torch.Tensor
               ) -> torch.Tensor:
        """QKV projection, RoPE + KV write, attention: [T, nq * d], the o_proj input."""
        meta = meta.for_layer(self.window)  # sliding-window layers: their own KV group's tables
        qkv = ops.linear(x, self.qkv_weight, self.qkv_bias)
        k_cache, v_cache = kv
        # under attention DP the slot mapping covers every replica's rows (-1 outside this
        # replica's), so only this replica's K/V reach its cache
        q = ops.rope_and_cache(qkv, positions, cos_sin, k_cache, v_cache, meta.slot_mapping, self.nq, self.nkv,
                               self.d, self.k_scale, self.v_scale)
        if self.adp is not None:
            q = self.adp.all_to_all(q.contiguous(), scatter_dim=0, gather_dim=1)  # own rows, TP-rank heads
        o = ops.attention(q, k_cache, v_cache, meta, self.scale, self.sinks, self.window, self.k_scale,
                          self.v_scale)
        if self.adp is not None:
            o = self.adp.all_to_all(o, scatter_dim=1, gather_dim=0)  # every row, this rank's q shard
        return o.reshape(o.shape[0], self.nq * self.d)


class GptOssExperts(nn.Module):
    """This rank's experts.  MXFP4: w13 [E_l, 2I, H/2] u8 + s13 [E_l, 2I, H/32] u8,
    w2 [E_l, H, I/2] + s2 [E_l, H, I/32]; bf16: w13 [E_l, 2I, H], w2 [E_l, H, I].

    Sharding (``model_mxfp4.py:879-911``, variable EP ``neuron_parallel_state.py:153-167``):
    ``ep_size`` partitions of ``E / ep_size`` experts; inside a partition the intermediate
    dimension is split over ``mtp_size`` ranks (MoE tensor parallelism), I padded with zero
    channels to a multiple of ``mtp_size`` x 32 (one MX scale block; 2880 -> 3072 at 8 ranks,
    the padding the reference uses) so every slice is whole scale blocks.  A zero channel
    contributes nothing: its gate and up are 0, SwiGLU(0, 0) = 0.  The down-projection bias
    is added by slice 0 only, so the partial sums over the ranks add it once."""

    def __init__(self, cfg: GptOssConfig, ep_rank: int, ep_size: int, dtype, device, mtp_rank: int = 0,
                 mtp_size: int = 1):
        super().__init__()
        E, H, I = cfg.num_local_experts, cfg.hidden_size, cfg.intermediate_size
        if E % ep_size:
            raise ValueError(f"{E} experts not divisible by ep {ep_size}")
        self.E_local = E // ep_size
        self.offset = ep_rank * self.E_local
        self.quant = cfg.quantization
        self.alpha, self.limit = cfg.swiglu_alpha, cfg.swiglu_limit
        self.mtp_rank, self.mtp_size = mtp_rank, mtp_size
        unit = (32 if self.quant == "mxfp4" else 8) * mtp_size
        self.I_full = I
        self.I_pad = round_up(I, unit) if mtp_size > 1 else I
        I_loc = self.I_pad // mtp_size
        self.i0 = mtp_rank * I_loc
        self.H, self.I = H, I_loc
        if self.quant == "mxfp4":
            if H % 32 or I_loc % 32:
                raise ValueError("MXFP4 needs hidden and (per-rank) intermediate sizes divisible by 32")
            # kernel layout (ops/mx_layout.py): 128x128 value tiles stored contiguously,
            # scales in 512-byte atoms
            k1, k2 = round_up(H, 128), round_up(I_loc, 128)
            self.w13 = _param(tiled_shape(self.E_local, 2 * I_loc, H), torch.uint8, device)
            self.s13 = _param((self.E_local, -(-2 * I_loc // 128), k1 // 128, 512), torch.uint8, device)
            self.w2 = _param(tiled_shape(self.E_local, H, I_loc), torch.uint8, device)
            self.s2 = _param((self.E_local, -(-H // 128), k2 // 128, 512), torch.uint8, device)
        else:
            self.w13 = _param((self.E_local, 2 * I_loc, H), dtype, device)
            self.w2 = _param((self.E_local, H, I_loc), dtype, device)
        self.b13 = _param((self.E_local, 2 * I_loc), torch.float32, device)
        self.b2 = _param((self.E_local, H), torch.float32, device)

    # -- slices of the (experts x intermediate) checkpoint tensors this rank holds ------------
    def slice_13(self, t: torch.Tensor, dim: int = 1) -> torch.Tensor:
        """Gate/up rows (interleaved 2i gate, 2i+1 up) of this rank's intermediate slice,
        zero rows for the padding."""
        if self.mtp_size == 1:
            return t
        return _pad_narrow(t, dim, 2 * self.I_full, 2 * self.I_pad, 2 * self.i0, 2 * self.I)

    def slice_2(self, t: torch.Tensor, dim: int, per: int = 1) -> torch.Tensor:
        """Down-projection K entries (``per`` elements each: 1 for values, 32 for MX blocks)
        of this rank's intermediate slice, zeros for the padding."""
        if self.mtp_size == 1:
            return t
        return _pad_narrow(t, dim, self.I_full // per, self.I_pad // per, self.i0 // per, self.I // per)

    def local(self, full: torch.Tensor) -> torch.Tensor:
        return full[self.offset:self.offset + self.E_local]

    def forward(self, x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        if self.quant == "mxfp4":
            return ops.moe_mxfp4(x, ids, w, self.w13, self.s13, self.b13, self.w2, self.s2, self.b2, self.offset,
                                 self.alpha, self.limit, self.H, self.I)
        return ops.moe_dense(x, ids, w, self.w13, self.b13, self.w2, self.b2, self.offset, self.alpha, self.limit,
                             True, "swiglu_clamp", self.H, self.I)

    @torch.no_grad()
    def process_weights_after_loading(self) -> None:
        """bf16 experts on a GPU: re-lay the weights into the grouped-GEMM tiles."""
        if self.quant != "mxfp4" and self.w13.is_cuda and self.w13.dim() == 3:
            t13, t2 = ops.prepare_moe_bf16(self.w13.data, self.w2.data, interleaved=True)
            self.w13 = nn.Parameter(t13, requires_grad=False)
            self.w2 = nn.Parameter(t2, requires_grad=False)


class GptOssMLP(nn.Module):
    """Experts are sharded over the whole world (EP = TP x DP).  With data parallelism the
    tokens of every replica are gathered over the DP group before the experts and the
    partial outputs reduce-scattered back (cross-DP EP, ``model_mxfp4.py:1361-1453``); the
    TP partial sum is completed at the next layer boundary."""

    def __init__(self, cfg: GptOssConfig, ps: ParallelState, dtype, device, rows_group: GroupCoordinator | None = None):
        super().__init__()
        self.cfg = cfg
        # rows are replicated over ``tp`` (the attention-DP supergroup when set: every DP
        # replica's tokens are already there, so no gather over DP)
        self.dp = ps.dp if rows_group is None else _single_group()
        self.tp = rows_group or ps.tp
        # expert partitions over the EP group, intermediate slices over the EP-TP group (ranks
        # of one partition); rank r = partition * (world / ep) + slice
        world = ps.tp.world_size * ps.dp.world_size
        ep_size = int(ps.degrees.get("ep", world)) if world > 1 else 1
        mtp_size = world // ep_size
        r = ps.dp.rank_in_group * ps.tp.world_size + ps.tp.rank_in_group
        ep_rank, mtp_rank = r // mtp_size, r % mtp_size
        self.router_weight = _param((cfg.num_local_experts, cfg.hidden_size), dtype, device)
        self.router_bias = _param((cfg.num_local_experts,), dtype, device)
        self.experts = GptOssExperts(cfg, ep_rank, ep_size, dtype, device, mtp_rank, mtp_size)
        # EP all-to-all (``parallel/all2all.py``), attached by the worker when
        # ``all2all_backend`` asks for one; None: all-gather / reduce-scatter over DP
        self.a2a = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """This rank's partial MoE output (its experts only); the caller reduces it."""
        if self.a2a is not None:
            # route the local tokens; each TP rank sends its slice to the expert owners
            # and gets their outputs back (zeros outside the slice: a TP partial sum)
            from ..parallel.all2all import ep_slice

            T = x.shape[0]
            ids, w = ops.router_topk(x, self.router_weight, self.router_bias, self.cfg.num_experts_per_tok)
            t0, t1 = ep_slice(T, self.tp.rank_in_group, self.tp.world_size)
            xr, ir, wr = self.a2a.dispatch(x, ids, w, self.experts.E_local, t0, t1)
            return self.a2a.combine(self.experts(xr, ir, wr), T)
        if self.dp.world_size > 1:
            x = self.dp.all_gather(x, dim=0)
        ids, w = ops.router_topk(x, self.router_weight, self.router_bias, self.cfg.num_experts_per_tok)
        if self._defer_route_sum(x):
            # the per-token sum over routes happens inside the layer-boundary all-reduce kernel
            ex = self.experts
            y = torch.empty(x.shape[0] * ids.shape[1], x.shape[1], dtype=x.dtype, device=x.device)
            ops.moe_mxfp4(x, ids, w, ex.w13, ex.s13, ex.b13, ex.w2, ex.s2, ex.b2, ex.offset, ex.alpha, ex.limit,
                          ex.H, ex.I, y_routes=y)
            return RoutePartial(y, ids, ex.E_local, ex.offset)
        y = self.experts(x, ids, w)
        return self.dp.reduce_scatter(y, dim=0) if self.dp.world_size > 1 else y

    def _defer_route_sum(self, x: torch.Tensor) -> bool:
        if not (envs.VLLM_B200_FUSE_MOE_ROUTE_SUM and x.is_cuda and self.dp.world_size == 1
                and self.tp.world_size > 1 and self.experts.quant == "mxfp4"):
            return False
        if self.tp.sp_active:  # the SP boundary kernel sums the routes while it scatters
            sc = self.tp.sp_comm
            return sc is not None and sc.can(x.shape[0], x.shape[1])
        comm = self.tp.communicator
        return comm is not None and comm.can_all_reduce(x)


class GptOssDecoderLayer(nn.Module):
    """Input: the previous layer's MoE partial sum (or the embedding for layer 0).  Each
    layer boundary is one ``all_reduce_add_rmsnorm``: reduce the partial sums across the
    group, add bias and residual, normalise."""

    def __init__(self, cfg: GptOssConfig, i: int, ps: ParallelState, dtype, device):
        super().__init__()
        self.eps = cfg.rms_norm_eps
        self.tp = ps.tp
        adp = _attention_dp(ps)
        if adp is not None:  # every layer boundary reduces over the attention-DP supergroup
            self.tp = ps.attn_tp
        self.moe_group = self.tp
        self.input_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps, device=device)
        self.self_attn = GptOssAttention(cfg, i, self.tp, dtype, device, adp)
        self.post_attention_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps, device=device)
        self.mlp = GptOssMLP(cfg, ps, dtype, device, rows_group=ps.attn_tp if adp is not None else None)

    def forward(self, positions, h, residual, meta, kv, cos_sin):
        if residual is None:
            residual = h
            x = self.input_layernorm(h)
        else:
            x, residual = self.moe_group.all_reduce_add_rmsnorm(h, residual, self.input_layernorm.weight, self.eps)
        # the output projection of this rank's heads, the all-reduce, bias, residual add and the
        # next RMSNorm: a GEMM that reduces through NVSwitch + one finish kernel, or the GEMM +
        # one fused all-reduce kernel
        a = self.self_attn.attend(positions, x, meta, kv, cos_sin)
        x, residual = self.tp.linear_all_reduce_add_rmsnorm(a, self.self_attn.o_proj.weight, residual,
                                                            self.post_attention_layernorm.weight, self.eps,
                                                            self.self_attn.o_proj.bias)
        return self.mlp(x), residual


class GptOssForCausalLM(nn.Module):
    """Model entry point used by the runner: ``forward`` returns the hidden states
    of the tokens selected by ``meta.logits_indices``; ``compute_logits`` returns this
    rank's vocab shard of the logits."""

    config_class = GptOssConfig

    def __init__(self, cfg: GptOssConfig, ps: ParallelState, dtype=torch.bfloat16, device="cpu",
                 kv_dtype: torch.dtype | None = None):
        super().__init__()
        self.cfg = cfg
        self.ps = ps
        self.dtype = dtype
        self.kv_dtype = kv_dtype or dtype
        adp = _attention_dp(ps)
        # the group whose ranks hold the same rows (TP, or the attention-DP supergroup)
        self.tp = ps.attn_tp if adp is not None else ps.tp
        emb = {"group": self.tp, "dp_group": None} if adp is not None else component(ps, "embedding")
        self.embed_tokens = VocabParallelEmbedding(cfg.vocab_size, cfg.hidden_size, dtype=dtype, device=device,
                                                   **emb)
        self.layers = nn.ModuleList([GptOssDecoderLayer(cfg, i, ps, dtype, device)
                                     for i in range(cfg.num_hidden_layers)])
        self.norm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps, device=device)
        # under attention DP the head is sharded over the supergroup and the runner samples
        # every replica's rows (as with lm_head DP)
        lmh = {"group": self.tp, "dp_group": adp} if adp is not None else component(ps, "lm_head")
        self.lm_head = ParallelLMHead(cfg.vocab_size, cfg.hidden_size, dtype=dtype, device=device, **lmh)
        self.attention_dp = adp
        inv, af = cfg.rope_params()
        self.register_buffer("cos_sin", ops.build_cos_sin_cache(inv, min(cfg.max_position_embeddings, 1 << 17),
                                                                af, device=device), persistent=False)
        self.aux_hidden_layers: tuple[int, ...] = ()

    # ------------------------------------------------------------------ spec
    def get_kv_spec(self) -> KVSpec:
        return KVSpec([LayerSpec(l.self_attn.nkv, self.cfg.head_dim, self.kv_dtype, l.self_attn.window)
                       for l in self.layers])

    def set_kv_scales(self, k_scale: float, v_scale: float) -> None:
        for l in self.layers:
            l.self_attn.k_scale, l.self_attn.v_scale = k_scale, v_scale

    # --------------------------------------------------------------- forward
    def forward(self, input_ids: torch.Tensor, positions: torch.Tensor, meta, kv_caches: list,
                inputs_embeds: torch.Tensor | None = None) -> torch.Tensor:
        h = self.embed_tokens(input_ids) if inputs_embeds is None else inputs_embeds
        residual = None
        aux = []
        for i, layer in enumerate(self.layers):
            if i in self.aux_hidden_layers:  # hidden state entering layer i (reduced partial + residual)
                if isinstance(h, RoutePartial):
                    h = h.materialize()
                aux.append(h if residual is None else self.tp.all_reduce(h.clone()) + residual)
            h, residual = layer(positions, h, residual, meta, kv_caches[i], self.cos_sin)
        h, _ = self.tp.all_reduce_add_rmsnorm(h, residual, self.norm.weight, self.cfg.rms_norm_eps)
        self._aux = torch.cat(aux, dim=-1) if aux else None
        return h

    def get_eagle3_aux_hidden_state_layers(self) -> tuple[int, ...]:
        """Low / middle / high layers feeding an EAGLE-3 draft (``model_mxfp4.py:2033-2037``)."""
        n = self.cfg.num_hidden_layers
        return (2, n // 2, n - 3) if n >= 8 else (0, n // 2, n - 1)

    def compute_logits(self, h: torch.Tensor) -> torch.Tensor:
        return self.lm_head(h)

    # ----------------------------------------------------------------- loading
    def load_weights(self, weights: Iterable[tuple[str, torch.Tensor]]) -> set[str]:
        """Consume (name, full tensor) pairs in the HF checkpoint naming, including the
        MXFP4 ``*_blocks``/``*_scales`` expert keys and the bf16 ``gate_up_proj``
        [E, H, 2I] / ``down_proj`` [E, I, H] layout."""
        loaded = set()
        for name, t in weights:
            n = name[len("model."):] if name.startswith("model.") else name
            if n == "embed_tokens.weight":
                self.embed_tokens.weight.weight_loader(self.embed_tokens.weight, t)
                if self.cfg.tie_word_embeddings:
                    self.lm_head.weight.weight_loader(self.lm_head.weight, t)
            elif n in ("lm_head.weight",) or name == "lm_head.weight":
                self.lm_head.weight.weight_loader(self.lm_head.weight, t)
            elif n == "norm.weight":
                self.norm.weight.data.copy_(t.float())
            elif n.startswith("layers."):
                parts = n.split(".")
                li = int(parts[1])
                rest = ".".join(parts[2:])
                self._load_layer(self.layers[li], rest, t)
            else:
                continue
            loaded.add(name)
        return loaded

    def _load_layer(self, layer: GptOssDecoderLayer, rest: str, t: torch.Tensor) -> None:
        at, mlp = layer.self_attn, layer.mlp
        ex = mlp.experts
        if rest in ("input_layernorm.weight", "post_attention_layernorm.weight"):
            getattr(layer, rest.split(".")[0]).weight.data.copy_(t.float())
        elif rest.startswith("self_attn.") and rest.split(".")[1] in ("q_proj", "k_proj", "v_proj"):
            which = rest.split(".")[1][0]
            at.load_q_k_v(which, rest.split(".")[2], t)
        elif rest == "self_attn.o_proj.weight":
            at.o_proj.weight.weight_loader(at.o_proj.weight, t)
        elif rest == "self_attn.o_proj.bias":
            at.o_proj.bias.data.copy_(t.to(at.o_proj.bias.dtype))
        elif rest == "self_attn.sinks":
            at.load_sinks(t)
        elif rest == "mlp.router.weight":
            mlp.router_weight.data.copy_(t.to(mlp.router_weight.dtype))
        elif rest == "mlp.router.bias":
            mlp.router_bias.data.copy_(t.to(mlp.router_bias.dtype))
        elif rest == "mlp.experts.gate_up_proj_bias":
            ex.b13.data.copy_(ex.slice_13(ex.local(t).float(), 1))
        elif rest == "mlp.experts.down_proj_bias":
            # added once: by the first intermediate slice of each partition
            ex.b2.data.copy_(ex.local(t).float() if ex.mtp_rank == 0 else torch.zeros_like(ex.b2))
        elif rest == "mlp.experts.gate_up_proj_blocks":
            self._load_mx(ex, "13", "blocks", t)
        elif rest == "mlp.experts.gate_up_proj_scales":
            self._load_mx(ex, "13", "scales", t)
        elif rest == "mlp.experts.down_proj_blocks":
            self._load_mx(ex, "2", "blocks", t)
        elif rest == "mlp.experts.down_proj_scales":
            self._load_mx(ex, "2", "scales", t)
        elif rest == "mlp.experts.gate_up_proj":  # bf16 [E, H, 2I]
            self._load_dense(ex, "13", ex.slice_13(ex.local(t).transpose(1, 2), 1))
        elif rest == "mlp.experts.down_proj":  # bf16 [E, I, H]
            self._load_dense(ex, "2", ex.slice_2(ex.local(t).transpose(1, 2), 2))
        else:
            raise KeyError(f"unexpected GPT-OSS weight {rest}")

    @staticmethod
    def _load_mx(ex: GptOssExperts, which: str, kind: str, t: torch.Tensor) -> None:
        loc = ex.local(t)
        # blocks [E, rows, K/32, 16], scales [E, rows, K/32]: gate/up rows or down K blocks
        # of this rank's intermediate slice
        loc = ex.slice_13(loc, 1) if which == "13" else ex.slice_2(loc, 2, 32)
        K = ex.H if which == "13" else ex.I
        if ex.quant == "mxfp4":
            if kind == "blocks":
                vals = loc.reshape(loc.shape[0], loc.shape[1], -1)
                getattr(ex, "w" + which).data.copy_(tile_values(vals.to(ex.w13.device), K))
            else:
                getattr(ex, "s" + which).data.copy_(scales_to_atoms(loc.to(ex.w13.device), K))
            return
        # bf16 model served from an MXFP4 checkpoint: dequantise at load time
        # (``weight_loaders_bf16.py:264``); needs the matching blocks/scales pair.
        pend = ex.__dict__.setdefault("_pending", {})
        pend[(which, kind)] = loc
        if (which, "blocks") in pend and (which, "scales") in pend:
            b = pend.pop((which, "blocks"))
            s = pend.pop((which, "scales"))
            GptOssForCausalLM._load_dense(ex, which, ref.dequant_mxfp4(b.reshape(*b.shape[:2], -1), s))

    @staticmethod
    def _load_dense(ex: GptOssExperts, which: str, w: torch.Tensor) -> None:
        if ex.quant == "mxfp4":
            K = ex.H if which == "13" else ex.I
            blocks, scales = ref.quantize_mxfp4(w.float())
            getattr(ex, "w" + which).data.copy_(tile_values(blocks, K))
            getattr(ex, "s" + which).data.copy_(scales_to_atoms(scales, K))
        else:
            getattr(ex, "w" + which).data.copy_(w.to(getattr(ex, "w" + which).dtype))
