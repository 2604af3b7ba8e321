"""Functional op library: hand-written sm_100a kernel on CUDA tensors, PyTorch
reference otherwise.

This is the B200 counterpart of the Trainium plugin's ``functional`` package
(``vllm_neuron/functional/__init__.py:42-74``), where each op chose an NKI kernel
or a PyTorch fallback.  Here the choice is simpler: a CUDA tensor runs the
compiled kernel (``torch.ops.b200.*``; a missing extension is an error), a CPU
tensor (or ``VLLM_B200_DISABLE_KERNELS=1``) runs :mod:`.reference`.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from . import reference as ref
from ._ext import kernels_enabled, use_kernel  # noqa: F401
from ._ext import ops as _k
from .metadata import AttentionMetadata
from .reference import deltanet as ref_dn  # noqa: F401

_STATUS: dict = {}


def device_status(device: torch.device) -> torch.Tensor:
    """Per-device int32 status word that kernels with bounded waits or index checks
    write (0 = ok; codes 1001.. as in ``csrc/common.cuh`` StatusCode, so they never
    collide with a ``cudaError_t``).  Read it with
    :func:`check_device_status` between steps."""
    key = str(device)
    t = _STATUS.get(key)
    if t is None:
        t = torch.zeros(4, dtype=torch.int32, device=device)  # code, where, value, spare
        _STATUS[key] = t
    return t


def check_device_status(device: torch.device) -> int:
    """Raise if a kernel on ``device`` recorded an error; returns the code (0)."""
    t = _STATUS.get(str(device))
    if t is None:
        return 0
    code, where, value, _ = t.tolist()
    if code:
        t.zero_()
        names = {1001: "index out of range", 1002: "device wait timed out", 1003: "bad shape",
                 1004: "bad alignment", 1005: "scratch too small"}
        raise RuntimeError(f"kernel status {code} ({names.get(code, 'unknown')}) at check {where}, value {value}")
    return 0

# ---------------------------------------------------------------------------
# dense layers
# ---------------------------------------------------------------------------


_GEMM_WS: dict = {}
_GEMM_MAX_SPLITS = 16


def _gemm_workspace(device: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-device split-K scratch of the dense GEMM: fp32 sums [T, N] of a call whose output
    tiles are fewer than the SMs (so at most one tile per SM) and one arrival counter per
    tile and epilogue warp; both are zero between calls (each call clears what it used).
    Allocated once, before any capture."""
    key = str(device)
    ws = _GEMM_WS.get(key)
    if ws is None:
        sms = torch.cuda.get_device_properties(device).multi_processor_count
        ws = (torch.zeros(sms * 128 * 256, dtype=torch.float32, device=device),
              torch.zeros(4 * max(256, sms), dtype=torch.int32, device=device))
        _GEMM_WS[key] = ws
    return ws


def _gemm_ok(x: torch.Tensor, w: torch.Tensor) -> bool:
    from .. import envs

    return (use_kernel(x) and w.dtype == torch.bfloat16 and w.dim() == 2 and w.is_contiguous()
            and w.shape[1] % 8 == 0 and w.shape[0] % 8 == 0 and not envs.VLLM_B200_LIBRARY_GEMM)


def linear(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None = None,
           out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """y = x . w^T + b.  bf16 on a GPU: the tcgen05 GEMM of ``csrc/gemm.cu`` (split K when
    the output tiles cannot fill the SMs); anything else: torch.  ``out_dtype=float32``
    keeps the fp32 accumulator (router logits).  Row-parallel projections whose sum is
    reduced across the TP group go through ``GroupCoordinator.linear_all_reduce_add_rmsnorm``."""
    if x.dtype != w.dtype:
        x = x.to(w.dtype)
    if _gemm_ok(x, w):
        K, N = w.shape[1], w.shape[0]
        x2 = x.reshape(-1, K)
        if x2.stride(1) != 1 or x2.stride(0) % 8 or x2.data_ptr() % 16:
            x2 = x2.contiguous()
        y = torch.empty(x2.shape[0], N, dtype=out_dtype or w.dtype, device=x.device)
        ws, cnt = _gemm_workspace(x.device)
        bb = b.to(w.dtype).contiguous() if b is not None else None
        _k().gemm_bf16(y, x2, w, bb, ws, cnt, _GEMM_MAX_SPLITS, device_status(x.device))
        return y.reshape(*x.shape[:-1], N)
    y = F.linear(x, w, b)
    return y.to(out_dtype) if out_dtype is not None else y


def gemm_available(x: torch.Tensor, w: torch.Tensor) -> bool:
    """The bf16 tcgen05 GEMM takes these operands (``linear`` would not fall back to torch)."""
    return x.dtype == torch.bfloat16 and _gemm_ok(x, w)


def linear_scatter(x: torch.Tensor, w: torch.Tensor, dst: list[int], ldd: int) -> None:
    """x . w^T (bf16, no bias) with the rows split into ``len(dst)`` equal blocks, block q
    stored from device address ``dst[q]`` with a row stride of ``ldd`` elements: the tcgen05
    GEMM of ``csrc/gemm.cu`` writing a sequence-parallel reduce-scatter's partial rows straight
    into their owners' receive areas (peer memory, plain stores from the epilogue)."""
    if not _gemm_ok(x, w) or x.dtype != torch.bfloat16:
        raise RuntimeError("linear_scatter needs the bf16 tcgen05 GEMM")
    x2 = x.reshape(-1, w.shape[1])
    if x2.stride(1) != 1 or x2.stride(0) % 8 or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    ws, cnt = _gemm_workspace(x.device)
    _k().gemm_scatter(list(dst), ldd, x2, w, ws, cnt, _GEMM_MAX_SPLITS, device_status(x.device))


def linear_fp8(x: torch.Tensor, w_fp8: torch.Tensor, w_scale: torch.Tensor, in_scale: torch.Tensor | None,
               b: torch.Tensor | None = None, x_q: torch.Tensor | None = None,
               alpha: torch.Tensor | None = None, out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """Static FP8 linear (ModelOpt checkpoints, ``model/llama3/quantization.py:176``):
    y = (q(x / s_in) @ W_fp8^T) * s_in * s_w, q = e4m3 with saturation; ``w_scale`` per
    tensor ([1]) or per output feature ([N], e.g. the q / k / v segments of a fused QKV).
    Dynamic per-tensor activation scale when ``in_scale`` is None.  On a GPU: the e4m3
    quantisation kernel (``csrc/fp8.cu``, which also writes alpha = s_in * s_w on the device)
    and the tcgen05 kind::f8f6f4 GEMM of ``csrc/gemm.cu``, which scales its fp32 accumulator
    by alpha.  ``x_q``: activations already quantised with ``in_scale`` (the fused RMSNorm +
    quantisation); ``alpha``: s_in * s_w precomputed for a static ``in_scale``."""
    K, N = w_fp8.shape[1], w_fp8.shape[0]
    ws_n = w_scale.numel()
    if (use_kernel(w_fp8) and w_fp8.dtype == torch.float8_e4m3fn and w_fp8.is_contiguous() and K % 16 == 0
            and N % 8 == 0 and ws_n in (1, N) and (x_q is not None or x.dtype == torch.bfloat16)):
        lead = (x_q if x_q is not None else x).shape[:-1]
        if x_q is None:
            x2 = x.reshape(-1, K)
            if x2.stride(1) != 1 or x2.stride(0) % 16 or x2.data_ptr() % 16:
                x2 = x2.contiguous()
            xq = torch.empty(x2.shape, dtype=torch.float8_e4m3fn, device=x.device)
            if in_scale is not None and alpha is not None:
                _k().fp8_quant(xq, x2, in_scale.float().reshape(1), None, None, None)
            else:
                alpha = torch.empty(ws_n, dtype=torch.float32, device=x.device)
                amax = None if in_scale is not None else torch.empty(1, dtype=torch.int32, device=x.device)
                _k().fp8_quant(xq, x2, in_scale.float().reshape(1) if in_scale is not None else None, amax,
                               w_scale.float().reshape(-1), alpha)
        else:
            xq = x_q.reshape(-1, K)
            if alpha is None:
                alpha = in_scale.float().reshape(1) * w_scale.float().reshape(-1)
        y = torch.empty(xq.shape[0], N, dtype=torch.bfloat16, device=w_fp8.device)
        wsp, cnt = _gemm_workspace(w_fp8.device)
        bb = b.to(torch.bfloat16).contiguous() if b is not None else None
        _k().gemm_fp8(y, xq, w_fp8, bb, alpha.reshape(-1), wsp, cnt, _GEMM_MAX_SPLITS, device_status(w_fp8.device))
        return y.reshape(*lead, N)
    if x_q is not None:
        x = (x_q.float() * in_scale.float()).to(out_dtype or torch.bfloat16)
    xs = in_scale if in_scale is not None else (x.abs().amax().float().clamp_min(1e-12) / 448.0).reshape(1)
    xq = (x.float() / xs.float()).clamp(-448, 448).to(torch.float8_e4m3fn)
    y = (xq.float() @ w_fp8.float().t()) * (xs.float() * w_scale.float().reshape(-1))
    y = y.to(x.dtype)
    return y + b if b is not None else y


def rms_norm_fp8(x: torch.Tensor, w: torch.Tensor, eps: float, in_scale: torch.Tensor,
                 residual: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor | None]:
    """The reference's rmsnorm_quant: (residual + x), its RMSNorm * w quantised to e4m3 with
    the static ``in_scale``.  Returns (e4m3 rows for ``linear_fp8(x_q=...)``, the new residual;
    on a GPU the residual buffer is updated in place)."""
    if use_kernel(x) and x.dtype == torch.bfloat16 and x.shape[-1] % 8 == 0 and x.shape[-1] <= 8192:
        x2 = x.reshape(-1, x.shape[-1]).contiguous()
        q = torch.empty(x2.shape, dtype=torch.float8_e4m3fn, device=x.device)
        _k().rms_norm_fp8(q, x2, residual, w.float().contiguous(), eps, in_scale.float().reshape(1))
        return q.reshape(x.shape), residual
    if residual is not None:
        residual = (x.float() + residual.float()).to(residual.dtype)
        x = residual
    y = (x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype)
    return (y.float() / in_scale.float()).clamp(-448, 448).to(torch.float8_e4m3fn), residual


def silu_and_mul(gu: torch.Tensor) -> torch.Tensor:
    """[T, 2I] (gate | up) -> silu(gate) * up."""
    if use_kernel(gu) and gu.dtype == torch.bfloat16:
        out = torch.empty(gu.shape[0], gu.shape[1] // 2, dtype=gu.dtype, device=gu.device)
        _k().silu_and_mul(out, gu)
        return out
    I = gu.shape[-1] // 2
    return (F.silu(gu[..., :I].float()) * gu[..., I:].float()).to(gu.dtype)


def embedding(ids: torch.Tensor, w: torch.Tensor, vocab_start: int = 0) -> torch.Tensor:
    """Rows of ``w`` for ids in ``[vocab_start, vocab_start + rows)``, zero elsewhere."""
    if use_kernel(w):
        out = torch.empty(ids.shape[0], w.shape[1], dtype=w.dtype, device=w.device)
        _k().embedding(out, ids, w, vocab_start)
        return out
    local = ids.long() - vocab_start
    valid = (local >= 0) & (local < w.shape[0])
    y = w[local.clamp(0, w.shape[0] - 1)]
    return y * valid[:, None].to(y.dtype)


# ---------------------------------------------------------------------------
# normalisation
# ---------------------------------------------------------------------------


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    if use_kernel(x):
        out = torch.empty_like(x)
        _k().rms_norm(out, x, w, eps)
        return out
    return ref.rms_norm(x, w, eps)


def fused_add_rms_norm(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float
                       ) -> tuple[torch.Tensor, torch.Tensor]:
    """Returns (norm(x + residual), x + residual).  On GPU the residual buffer is
    updated in place."""
    if use_kernel(x):
        out = torch.empty_like(x)
        _k().fused_add_rms_norm(out, x, residual, w, eps)
        return out, residual
    return ref.fused_add_rms_norm(x, residual, w, eps)


# ---------------------------------------------------------------------------
# rotary + KV cache write
# ---------------------------------------------------------------------------


def rope_and_cache(qkv: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor, k_cache: torch.Tensor,
                   v_cache: torch.Tensor, slot_mapping: torch.Tensor, num_q: int, num_kv: int, head_dim: int,
                   k_scale: float = 1.0, v_scale: float = 1.0, q_norm_w: torch.Tensor | None = None,
                   k_norm_w: torch.Tensor | None = None, norm_eps: float = 1e-6,
                   rotary_dim: int | None = None) -> torch.Tensor:
    """Apply RoPE to q and k of the fused projection ``qkv [T, (num_q+2*num_kv)*d]``
    in place, write k and v to the paged cache, return the q view [T, num_q, d].

    ``cos_sin`` [max_pos, rotary_dim] fp32 holds cos in the first half, sin in the
    second (attention factor folded in).  Optional per-head RMSNorm of q/k before the
    rotation (Qwen3 QK-norm).  ``rotary_dim`` < d rotates only the leading dims
    (partial rotary, Qwen3-Next)."""
    T = qkv.shape[0]
    rd = rotary_dim or head_dim
    if use_kernel(qkv):
        _k().rope_kv_write(qkv, positions, cos_sin, k_cache, v_cache, slot_mapping, num_q, num_kv, head_dim,
                           rd, k_scale, v_scale, q_norm_w, k_norm_w, norm_eps)
        return qkv[:, : num_q * head_dim].view(T, num_q, head_dim)
    q = qkv[:, : num_q * head_dim].view(T, num_q, head_dim)
    k = qkv[:, num_q * head_dim:(num_q + num_kv) * head_dim].view(T, num_kv, head_dim)
    v = qkv[:, (num_q + num_kv) * head_dim:(num_q + 2 * num_kv) * head_dim].view(T, num_kv, head_dim)
    if q_norm_w is not None:
        q.copy_(ref.rms_norm(q, q_norm_w, norm_eps))
        k.copy_(ref.rms_norm(k, k_norm_w, norm_eps))
    pos = positions.long()
    cs = cos_sin[pos]
    cos, sin = cs[:, : rd // 2], cs[:, rd // 2:]
    if rd == head_dim:
        q.copy_(ref.apply_rope(q, cos, sin))
        k.copy_(ref.apply_rope(k, cos, sin))
    else:
        q[..., :rd] = ref.apply_rope(q[..., :rd], cos, sin)
        k[..., :rd] = ref.apply_rope(k[..., :rd], cos, sin)
    ref.write_kv_cache(k, v, k_cache, v_cache, slot_mapping, k_scale, v_scale)
    return q


def build_cos_sin_cache(inv_freq: torch.Tensor, max_pos: int, attn_factor: float = 1.0,
                        device=None) -> torch.Tensor:
    pos = torch.arange(max_pos, dtype=torch.float32, device=device)
    cos, sin = ref.rope_cos_sin(pos, inv_freq.to(device), attn_factor)
    return torch.cat([cos, sin], dim=-1).contiguous()


# ---------------------------------------------------------------------------
# attention
# ---------------------------------------------------------------------------


def mla_decode(q: torch.Tensor, cache: torch.Tensor, block_tables: torch.Tensor, seq_lens: torch.Tensor,
               scale: float, num_splits: int | None = None, max_seq_len: int | None = None) -> torch.Tensor:
    """Multi-head latent attention decode (absorbed form): q [B, Hq, 576] against the paged
    latent cache [num_blocks, block_size, 576] (512 latent + 64 rope dims, shared by all
    heads), output [B, Hq, 512].  On a GPU: the tcgen05 kernel of ``csrc/mla_decode.cu``
    (keys as the MMA's 128-row dimension, S and O in tensor memory, split-KV with a
    log-sum-exp merge); elsewhere the fp32 reference.  ``num_splits`` defaults to enough
    splits of each sequence's 128-key tiles to put one CTA on every SM (``max_seq_len``, if
    given, caps it without reading ``seq_lens`` on the host)."""
    B, Hq = q.shape[0], q.shape[1]
    if not (use_kernel(q) and q.dtype == torch.bfloat16 and cache.dtype == torch.bfloat16):
        return ref.attention.mla_decode(q, cache, block_tables, seq_lens, scale)
    if num_splits is None:
        sms = torch.cuda.get_device_properties(q.device).multi_processor_count
        groups = -(-Hq // 64) if Hq > 32 else 1
        num_splits = max(1, min(64, sms // max(1, B * groups)))
        if max_seq_len is not None:
            num_splits = max(1, min(num_splits, -(-max_seq_len // 128)))
    q = q.contiguous()
    out = torch.empty(B, Hq, 512, dtype=torch.bfloat16, device=q.device)
    ws = torch.empty(B * Hq * num_splits * 513, dtype=torch.float32, device=q.device) if num_splits > 1 else None
    _k().mla_decode(out, q, cache.contiguous(), block_tables.to(torch.int32).contiguous(),
                    seq_lens.to(torch.int32).contiguous(), float(scale), ws, num_splits, device_status(q.device))
    return out


def attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, meta: AttentionMetadata,
              scale: float, sinks: torch.Tensor | None = None, window: int | None = None,
              k_scale: float = 1.0, v_scale: float = 1.0, out: torch.Tensor | None = None) -> torch.Tensor:
    """Attention of this step's queries (already RoPE'd, their K/V already in the
    cache) over the paged cache.  q [T, Hq, d] (may be a strided view)."""
    T, Hq, d = q.shape
    win = int(window or 0)
    if meta.cp_group is not None:  # decode context parallelism: shard attention + merge over the group
        from ..parallel.dcp import dcp_attention

        o = dcp_attention(q, k_cache, v_cache, meta, scale, sinks, window, k_scale, v_scale)
        if out is not None:
            out.copy_(o)
            return out
        return o
    if use_kernel(q):
        if out is None:
            out = torch.empty(T, Hq, d, dtype=q.dtype, device=q.device)
        if meta.is_decode:
            _k().paged_attention_decode(out, q, k_cache, v_cache, meta.block_tables, meta.seq_lens, sinks, win,
                                        scale, k_scale, v_scale, meta.workspace, meta.num_splits)
        elif 0 < meta.num_decode_seqs < meta.num_seqs:
            # mixed step: the decode kernel for the single-token sequences (rows 0 .. D-1), the
            # prefill kernel for the prompt chunks (their query-start offsets index q directly)
            D = meta.num_decode_seqs
            _k().paged_attention_decode(out[:D], q[:D], k_cache, v_cache, meta.block_tables[:D], meta.seq_lens[:D],
                                        sinks, win, scale, k_scale, v_scale, meta.workspace, meta.num_splits)
            _k().paged_attention_prefill(out, q, k_cache, v_cache, meta.block_tables[D:], meta.seq_lens[D:],
                                         meta.query_start_loc[D:], sinks, win, scale, k_scale, v_scale,
                                         meta.max_query_len)
        else:
            _k().paged_attention_prefill(out, q, k_cache, v_cache, meta.block_tables, meta.seq_lens,
                                         meta.query_start_loc, sinks, win, scale, k_scale, v_scale,
                                         meta.max_query_len)
        return out
    o = ref.paged_attention(q, k_cache, v_cache, meta.block_tables, meta.seq_lens, meta.query_start_loc, scale,
                            sinks, window, k_scale, v_scale)
    if out is not None:
        out.copy_(o)
        return out
    return o


def attention_shard(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, meta: AttentionMetadata,
                    scale: float, window: int | None, k_scale: float, v_scale: float, cp_rank: int,
                    cp_size: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Attention of one decode-context-parallel shard over the tokens its cache holds
    (token t lives on rank ``(t // block_size) % cp_size``).  Returns the shard's normalised
    output [T, Hq, d] and natural-log LSE [T, Hq] fp32 (-inf where it holds no visible key);
    no sinks (they join once, in the merge)."""
    T, Hq, d = q.shape
    win = int(window or 0)
    if use_kernel(q):
        out = torch.empty(T, Hq, d, dtype=q.dtype, device=q.device)
        lse = torch.empty(T, Hq, dtype=torch.float32, device=q.device)
        if meta.is_decode:
            _k().paged_attention_decode_cp(out, lse, q, k_cache, v_cache, meta.block_tables, meta.seq_lens, win,
                                           scale, k_scale, v_scale, meta.workspace, meta.num_splits, cp_rank,
                                           cp_size)
        else:
            _k().paged_attention_prefill_cp(out, lse, q, k_cache, v_cache, meta.block_tables, meta.seq_lens,
                                            meta.query_start_loc, win, scale, k_scale, v_scale,
                                            meta.max_query_len, cp_rank, cp_size)
        return out, lse
    o, lse = ref.paged_attention(q, k_cache, v_cache, meta.block_tables, meta.seq_lens, meta.query_start_loc, scale,
                                 None, window, k_scale, v_scale, return_lse=True, cp_rank=cp_rank, cp_size=cp_size)
    return o, lse.transpose(0, 1).contiguous()


def varlen_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens: torch.Tensor, scale: float,
                     causal: bool = True, max_seqlen: int = 0) -> torch.Tensor:
    """Self attention over packed sequences without a cache (vision encoder)."""
    if use_kernel(q):
        out = torch.empty_like(q)
        _k().varlen_attention(out, q, k, v, cu_seqlens, scale, causal, int(max_seqlen))
        return out
    return ref.prefill_attention(q, k, v, cu_seqlens, scale, None, None, causal)


# ---------------------------------------------------------------------------
# MoE
# ---------------------------------------------------------------------------


def router_topk(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None, top_k: int,
                order: str = "topk_softmax") -> tuple[torch.Tensor, torch.Tensor]:
    """(topk_ids [T,k] int32, topk_weights [T,k] fp32)."""
    if use_kernel(x) and order in ("topk_softmax", "softmax_topk", "softmax_topk_unnormalized") \
            and w.shape[0] <= 1024 and top_k <= 16:
        # fp32 logits straight from the GEMM accumulator (the reference's router linear runs
        # in fp32, model_mxfp4.py:949-955): bf16-rounded logits would reorder near ties.
        # softmax -> top-k -> renormalise selects and weighs exactly as top-k -> softmax (the
        # softmax is monotonic and the renormalisation cancels its denominator); without the
        # renormalisation the kernel divides by the softmax denominator over all experts.
        logits = linear(x, w, b, out_dtype=torch.float32)
        ids = torch.empty(x.shape[0], top_k, dtype=torch.int32, device=x.device)
        wts = torch.empty(x.shape[0], top_k, dtype=torch.float32, device=x.device)
        _k().topk_softmax(ids, wts, logits, 1 if order == "softmax_topk_unnormalized" else 0)
        return ids, wts
    ref_order, renorm = ("softmax_topk", False) if order == "softmax_topk_unnormalized" else (order, True)
    ids, wts, _ = ref.router_topk(x, w, b, top_k, ref_order, renormalize=renorm)
    return ids.to(torch.int32), wts


def moe_mxfp4(x: torch.Tensor, topk_ids: torch.Tensor, topk_w: torch.Tensor, w13: torch.Tensor,
              s13: torch.Tensor, b13: torch.Tensor | None, w2: torch.Tensor, s2: torch.Tensor,
              b2: torch.Tensor | None, expert_offset: int, alpha: float, limit: float, H: int, I: int,
              status: torch.Tensor | None = None, fp4: bool = True,
              y_routes: torch.Tensor | None = None) -> torch.Tensor:
    """Routed experts with packed MX weights in the kernel layout (``ops/mx_layout.py``):
    w13 tiles [E_local, 2I/128, K1p/128, 128, 64] u8 (gate/up interleaved rows) + s13
    scale atoms, w2 tiles [E_local, H/128, K2p/128, 128, 64] + s2 atoms; biases fp32
    [E_local, 2I] / [E_local, H].
    Returns this rank's partial sum over its experts, [T, H] in x.dtype; with ``y_routes``
    ([T * k, H] bf16, GPU only) the per-route rows are left there unsummed and it is returned
    (the layer-boundary all-reduce sums them)."""
    E = w13.shape[0]
    if use_kernel(x) and x.dtype == torch.bfloat16:
        out = torch.empty_like(x) if y_routes is None else x
        b13_ = b13 if b13 is not None else torch.zeros(E, 2 * I, dtype=torch.float32, device=x.device)
        b2_ = b2 if b2 is not None else torch.zeros(E, H, dtype=torch.float32, device=x.device)
        st = status if status is not None else device_status(x.device)
        _k().moe_mx(out, x.contiguous(), topk_ids.to(torch.int32).contiguous(), topk_w.float().contiguous(), w13,
                    s13, b13_, w2, s2, b2_, expert_offset, H, I, fp4, alpha, limit, st, y_routes)
        return out if y_routes is None else y_routes
    from .mx_layout import atoms_to_scales, untile_values

    if fp4:
        w13f = ref.dequant_mxfp4(untile_values(w13, 2 * I, H), atoms_to_scales(s13, 2 * I, H))
        w2f = ref.dequant_mxfp4(untile_values(w2, H, I), atoms_to_scales(s2, H, I))
    else:
        w13f = ref.dequant_mxfp8(untile_values(w13, 2 * I, H, False).view(torch.float8_e4m3fn),
                                 atoms_to_scales(s13, 2 * I, H))
        w2f = ref.dequant_mxfp8(untile_values(w2, H, I, False).view(torch.float8_e4m3fn), atoms_to_scales(s2, H, I))
    act = "swiglu_clamp" if limit is not None and limit > 0 else "silu"
    return ref.moe_experts(x, topk_ids, topk_w, w13f, b13, w2f, b2, alpha, limit if limit and limit > 0 else None,
                           True, expert_offset, act)


def prepare_moe_mxfp8(w13: torch.Tensor, w2: torch.Tensor, interleaved: bool) -> tuple[torch.Tensor, ...]:
    """Expert weights (any float dtype) -> MXFP8 kernel layout: e4m3 values with one ue8m0 scale
    per row and 32 K-elements, tiled [E, rows/128, Kp/128, 128, 128] u8 + 512-byte scale atoms.
    Used for fp8 checkpoints: block-scaled (128 x 128) fp8 weights are re-expressed with
    power-of-two scales per 32 elements, which the tensor cores apply in the MMA itself."""
    from .mx_layout import interleave_gate_up, scales_to_atoms, tile_values

    w13i = w13 if interleaved else interleave_gate_up(w13)
    out = []
    for w in (w13i, w2):
        K = w.shape[-1]
        q, sc = ref.quantize_mxfp8(w.float())
        out += [tile_values(q.view(torch.uint8), K, fp4=False), scales_to_atoms(sc, K)]
    return tuple(out)


def moe_dense(x: torch.Tensor, topk_ids: torch.Tensor, topk_w: torch.Tensor, w13: torch.Tensor,
              b13: torch.Tensor | None, w2: torch.Tensor, b2: torch.Tensor | None, expert_offset: int,
              alpha: float, limit: float | None, interleaved: bool = True, act: str = "swiglu_clamp",
              H: int | None = None, I: int | None = None) -> torch.Tensor:
    """Routed experts with bf16 weights.  Reference layout: w13 [E, 2I, H], w2 [E, H, I]
    (gate/up interleaved or halves).  Kernel layout (``prepare_moe_bf16``): tiles
    w13 [E, 2I/128, Hp/64, 128, 64] with gate/up interleaved, w2 [E, H/128, Ip/64, 128, 64];
    ``H`` and ``I`` must then be given.  ``act``: "swiglu_clamp" (GPT-OSS, alpha/limit) or
    "silu" (SiLU(gate) * up)."""
    if w13.dim() == 5:
        if not use_kernel(x):
            raise RuntimeError("tiled bf16 expert weights need the CUDA kernels")
        E = w13.shape[0]
        out = torch.empty_like(x)
        b13_ = b13 if b13 is not None else _zeros_f32(E * 2 * I, x.device)
        b2_ = b2 if b2 is not None else _zeros_f32(E * H, x.device)
        lim = float(limit) if (act == "swiglu_clamp" and limit is not None) else -1.0
        _k().moe_bf16(out, x.contiguous(), topk_ids.to(torch.int32).contiguous(), topk_w.float().contiguous(), w13,
                      b13_, w2, b2_, expert_offset, H, I, alpha if act == "swiglu_clamp" else 1.0, lim,
                      device_status(x.device))
        return out
    return ref.moe_experts(x, topk_ids, topk_w, w13, b13, w2, b2, alpha, limit, interleaved, expert_offset, act)


_ZEROS: dict = {}


def _zeros_f32(n: int, device) -> torch.Tensor:
    key = (str(device), n)
    z = _ZEROS.get(key)
    if z is None:
        z = _ZEROS[key] = torch.zeros(n, dtype=torch.float32, device=device)
    return z


def prepare_moe_bf16(w13: torch.Tensor, w2: torch.Tensor, interleaved: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """Reference-layout bf16 experts -> the kernel's tiled layout (gate/up interleaved)."""
    from .mx_layout import interleave_gate_up, tile_bf16

    w13i = w13 if interleaved else interleave_gate_up(w13)
    return tile_bf16(w13i.to(torch.bfloat16)), tile_bf16(w2.to(torch.bfloat16))


# ---------------------------------------------------------------------------
# gated DeltaNet (Qwen3-Next linear attention) and gating helpers
# ---------------------------------------------------------------------------


def _state_meta(meta: AttentionMetadata):
    ex = meta.extras
    return meta.query_start_loc, ex["state_slots"], ex["state_init"]


def causal_conv1d(x: torch.Tensor, w: torch.Tensor, conv_state: torch.Tensor, meta: AttentionMetadata
                  ) -> torch.Tensor:
    """Depthwise causal conv (kernel K) + SiLU per sequence, continuing from / updating the
    per-slot conv state [slots, C, K-1].  x [T, C] may be a row-strided view."""
    qsl, slots, init = _state_meta(meta)
    if use_kernel(x):
        out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
        _k().causal_conv1d(out, x, w, conv_state, qsl, slots, init, int(meta.max_query_len))
        return out
    return ref_dn.causal_conv1d(x, w, conv_state, qsl, slots, init)


def gated_delta_net(mixed: torch.Tensor, z: torch.Tensor, b: torch.Tensor, a: torch.Tensor, A_log: torch.Tensor,
                    dt_bias: torch.Tensor, norm_w: torch.Tensor, eps: float, state: torch.Tensor,
                    meta: AttentionMetadata, nk: int, nv: int, dk: int, dv: int) -> torch.Tensor:
    """Gated delta rule over the conv output ``mixed`` [T, 2*nk*dk + nv*dv] (q | k | v), with
    decay/strength from a, b [T, nv], followed by the per-head gated RMSNorm with z
    [T, nv*dv].  Continues from / updates the per-slot state [slots, nv, dk, dv] fp32.
    Returns [T, nv*dv] in mixed.dtype."""
    qsl, slots, init = _state_meta(meta)
    T = mixed.shape[0]
    if use_kernel(mixed):
        out = torch.empty(T, nv * dv, dtype=mixed.dtype, device=mixed.device)
        _k().gated_delta_net(out, mixed, z, b, a, A_log, dt_bias, norm_w, float(eps), state, qsl, slots, init,
                             nk, nv, dk, dv, bool(meta.is_decode), int(meta.max_query_len),
                             meta.extras.get("gdn_workspace"))
        return out
    q = mixed[:, :nk * dk].reshape(T, nk, dk)
    k = mixed[:, nk * dk:2 * nk * dk].reshape(T, nk, dk)
    v = mixed[:, 2 * nk * dk:].reshape(T, nv, dv)
    g, beta = ref_dn.gate_and_beta(a, b, A_log, dt_bias)
    o = ref_dn.gated_delta_rule(q, k, v, g, beta, state, qsl, slots, init)
    y = ref_dn.gated_rms_norm(o.to(mixed.dtype), z.reshape(T, nv, dv), norm_w, eps)
    return y.reshape(T, nv * dv)


def sigmoid_gate_mul(x: torch.Tensor, gate: torch.Tensor) -> torch.Tensor:
    """x * sigmoid(gate) elementwise (gate may be a row-strided view)."""
    if use_kernel(x):
        out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
        _k().sigmoid_gate_mul(out, x, gate)
        return out
    return (x.float() * torch.sigmoid(gate.float())).to(x.dtype)


def gated_add(x: torch.Tensor, y: torch.Tensor, gate_logit: torch.Tensor) -> torch.Tensor:
    """x + sigmoid(gate_logit) * y, gate_logit [T, 1] (shared-expert gate)."""
    if use_kernel(x):
        out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
        _k().gated_add(out, x, y, gate_logit)
        return out
    return (x.float() + torch.sigmoid(gate_logit.float()) * y.float()).to(x.dtype)


# ---------------------------------------------------------------------------
# sampling
# ---------------------------------------------------------------------------


def sample(logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor, top_p: torch.Tensor,
           uniform: torch.Tensor, max_top_k: int = 256) -> torch.Tensor:
    """One token per row.  temperature <= 0 -> greedy.  ``uniform`` [B] in [0,1)
    drives inverse-CDF sampling so that every TP rank draws the same token."""
    if use_kernel(logits):
        out = torch.empty(logits.shape[0], dtype=torch.int64, device=logits.device)
        _k().sample(out, logits, temperature, top_k, top_p, uniform, max_top_k)
        return out
    return ref.sample(logits, temperature, top_k, top_p, max_top_k=max_top_k, uniform=uniform)


def argmax(logits: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(max value fp32 [B], index int64 [B]) per row."""
    if use_kernel(logits):
        vals = torch.empty(logits.shape[0], dtype=torch.float32, device=logits.device)
        idx = torch.empty(logits.shape[0], dtype=torch.int64, device=logits.device)
        _k().argmax(vals, idx, logits)
        return vals, idx
    v, i = logits.float().max(-1)
    return v, i


def softmax_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)
