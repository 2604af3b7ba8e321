"""Attention references.

Semantics restated from the Trainium plugin's fallbacks:
* sink logits join the softmax denominator only (``functional/attention/attention_cte.py:163-173``,
  ``attention_decode.py:707-724``);
* a sliding window W lets query position p see keys j with p - W < j <= p
  (the HF mask ``kv_idx > q_idx - sliding_window``);
* FP8 KV is dequantised as ``k = k_fp8 * k_scale`` (``model_mxfp4.py:801,808`` fold the
  same scales into the softmax scale / W_out);
* the paged cache layout is HND: ``[num_blocks, kv_heads, block_size, head_dim]`` per
  layer for K and V (``vllm/attention/attn.py:27-35``); ``slot = block * block_size + offset``
  and a negative slot means "padding, do not write".
"""

from __future__ import annotations

import torch


def _softmax_with_sink(scores: torch.Tensor, sink: torch.Tensor | None) -> torch.Tensor:
    """scores [..., H, Q, K] fp32 with -inf masked; sink [H] or None."""
    if sink is None:
        m = scores.amax(-1, keepdim=True)
        m = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
        e = torch.exp(scores - m)
        return e / e.sum(-1, keepdim=True).clamp_min(1e-30)
    s = sink.float().view(*([1] * (scores.dim() - 3)), -1, 1, 1).expand(*scores.shape[:-1], 1)
    full = torch.cat([scores, s], dim=-1)
    m = full.amax(-1, keepdim=True)
    e = torch.exp(full - m)
    p = e / e.sum(-1, keepdim=True)
    return p[..., :-1]


def _attend(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_pos: torch.Tensor, k_pos: torch.Tensor,
            scale: float, sink: torch.Tensor | None, window: int | None, causal: bool = True,
            bounds: tuple[torch.Tensor, torch.Tensor] | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """q [Q, Hq, d], k/v [K, Hkv, d] -> (out [Q, Hq, d] fp32, lse [Hq, Q] fp32)."""
    hq, hkv = q.shape[1], k.shape[1]
    g = hq // hkv
    kf = k.float().repeat_interleave(g, dim=1)
    vf = v.float().repeat_interleave(g, dim=1)
    scores = torch.einsum("qhd,khd->hqk", q.float(), kf) * scale
    mask = torch.ones(q_pos.shape[0], k_pos.shape[0], dtype=torch.bool, device=q.device)
    if causal:
        mask &= k_pos[None, :] <= q_pos[:, None]
    if window is not None and window > 0:
        mask &= k_pos[None, :] > (q_pos[:, None] - window)
    if bounds is not None:
        lo, hi = bounds  # per-query [lo, hi) visible key index range (vision block packing)
        kidx = torch.arange(k_pos.shape[0], device=q.device)
        mask &= (kidx[None, :] >= lo[:, None]) & (kidx[None, :] < hi[:, None])
    scores = scores.masked_fill(~mask[None], float("-inf"))
    p = _softmax_with_sink(scores, sink)
    out = torch.einsum("hqk,khd->qhd", p, vf)
    m = scores.amax(-1)
    lse = torch.where(torch.isfinite(m), torch.logsumexp(scores, -1), torch.full_like(m, float("-inf")))
    return out, lse


def prefill_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens: torch.Tensor, scale: float,
                      sinks: torch.Tensor | None = None, sliding_window: int | None = None,
                      causal: bool = True, return_lse: bool = False):
    """Varlen self attention over packed sequences (``attention_cte.py:46``).

    q [T, Hq, d]; k, v [T, Hkv, d]; cu_seqlens [B+1] int."""
    out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    lse = torch.empty(q.shape[1], q.shape[0], dtype=torch.float32, device=q.device)
    cu = cu_seqlens.tolist()
    for b in range(len(cu) - 1):
        s, e = cu[b], cu[b + 1]
        if e == s:
            continue
        pos = torch.arange(e - s, device=q.device)
        o, l = _attend(q[s:e], k[s:e], v[s:e], pos, pos, scale, sinks, sliding_window, causal)
        out[s:e] = o
        lse[:, s:e] = l
    out = out.to(q.dtype)
    return (out, lse) if return_lse else out


def gather_kv_from_cache(k_cache: torch.Tensor, v_cache: torch.Tensor, block_table: torch.Tensor, length: int,
                         k_scale: float = 1.0, v_scale: float = 1.0) -> tuple[torch.Tensor, torch.Tensor]:
    """Materialise the first ``length`` tokens of one sequence: -> [length, Hkv, d] fp32."""
    bs = k_cache.shape[2]
    nblk = (length + bs - 1) // bs
    blocks = block_table[:nblk].long()
    k = k_cache[blocks].float().permute(0, 2, 1, 3).reshape(nblk * bs, k_cache.shape[1], -1)[:length]
    v = v_cache[blocks].float().permute(0, 2, 1, 3).reshape(nblk * bs, v_cache.shape[1], -1)[:length]
    return k * k_scale, v * v_scale


def paged_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_tables: torch.Tensor,
                    seq_lens: torch.Tensor, query_start_loc: torch.Tensor, scale: float,
                    sinks: torch.Tensor | None = None, sliding_window: int | None = None,
                    k_scale: float = 1.0, v_scale: float = 1.0, return_lse: bool = False,
                    cp_rank: int = 0, cp_size: int = 1):
    """Attention of new queries over a paged KV cache that already holds them.

    Sequence b owns query rows ``query_start_loc[b]:query_start_loc[b+1]`` (decode: 1
    row) at positions ``seq_lens[b] - q_len + i`` and attends keys ``[0, seq_lens[b])``
    causally.  This one definition covers decode (``attention_decode.py:354``),
    segmented/chunked prefill and prefix-cache hits (``attention_segmented_cte.py:103``).
    With ``cp_size > 1`` the cache is one decode-context-parallel shard: it holds the
    tokens t with ``(t // block_size) % cp_size == cp_rank``, densely, and the result is
    that shard's partial (sinks must be None; they join in :func:`lse_merge`).  Sequence
    lengths and windows stay global (``neuron_model_runner.py:279-328`` deals tokens the
    same way with ``cp_kv_cache_interleave_size = block_size``)."""
    out = torch.zeros(q.shape, dtype=torch.float32, device=q.device)
    lse = torch.full((q.shape[1], q.shape[0]), float("-inf"), dtype=torch.float32, device=q.device)
    qs = query_start_loc.tolist()
    sl = seq_lens.tolist()
    for b in range(len(sl)):
        s, e = qs[b], qs[b + 1]
        if e == s or sl[b] == 0:
            continue
        L = sl[b]
        bs = k_cache.shape[2]
        n_loc = cp_count_local(L, bs, cp_rank, cp_size)
        if n_loc == 0:
            continue
        k, v = gather_kv_from_cache(k_cache, v_cache, block_tables[b], n_loc, k_scale, v_scale)
        kpos = cp_global_pos(torch.arange(n_loc, device=q.device), bs, cp_rank, cp_size)
        qpos = torch.arange(L - (e - s), L, device=q.device)
        o, l = _attend(q[s:e], k, v, qpos, kpos, scale, sinks, sliding_window, True)
        out[s:e] = o
        lse[:, s:e] = l
    out = out.to(q.dtype)
    return (out, lse) if return_lse else out


def cp_count_local(x: int, block_size: int, cp_rank: int, cp_size: int) -> int:
    """How many of the global positions [0, x) belong to DCP rank ``cp_rank``."""
    if cp_size == 1:
        return x
    span = block_size * cp_size
    full, rem = divmod(x, span)
    return full * block_size + min(max(rem - cp_rank * block_size, 0), block_size)


def cp_global_pos(u, block_size: int, cp_rank: int, cp_size: int):
    """Global position of local token ``u`` (int or tensor) on DCP rank ``cp_rank``."""
    if cp_size == 1:
        return u
    return ((u // block_size) * cp_size + cp_rank) * block_size + u % block_size


def cp_slot_mapping(positions: torch.Tensor, block_tables: torch.Tensor, req_index: torch.Tensor,
                    block_size: int, cp_rank: int, cp_size: int) -> torch.Tensor:
    """Cache slots of new tokens on DCP rank ``cp_rank``: the owner writes token t at local
    index ``(t // (bs * cp)) * bs + t % bs`` of virtual block ``t // (bs * cp)``; every
    other rank gets -1 (skip)."""
    span = block_size * cp_size
    blk = block_tables[req_index.long(), (positions // span).long()].long()
    own = (positions // block_size) % cp_size == cp_rank
    slot = blk * block_size + positions % block_size
    return torch.where(own, slot, torch.full_like(slot, -1))


def write_kv_cache(k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                   slot_mapping: torch.Tensor, k_scale: float = 1.0, v_scale: float = 1.0) -> None:
    """Scatter new K/V rows [T, Hkv, d] into the HND paged cache at ``slot_mapping``
    (``functional/attention/qkv.py:296``).  Negative slots are skipped."""
    bs = k_cache.shape[2]
    valid = slot_mapping >= 0
    slots = slot_mapping[valid].long()
    blk, off = slots // bs, slots % bs
    kk, vv = k[valid], v[valid]
    if k_cache.dtype == torch.float8_e4m3fn:
        kk = (kk.float() / k_scale).clamp(-448, 448)
        vv = (vv.float() / v_scale).clamp(-448, 448)
    k_cache[blk, :, off] = kk.to(k_cache.dtype)
    v_cache[blk, :, off] = vv.to(v_cache.dtype)


def lse_merge(outs: list[torch.Tensor], lses: list[torch.Tensor],
              sink: torch.Tensor | None = None) -> torch.Tensor:
    """Combine partial attentions over disjoint key sets (split-KV / DCP).

    outs[i] [Q, H, d] are normalised partial outputs, lses[i] [H, Q] their
    log-sum-exp; the sink (if any) is added once to the global denominator."""
    L = torch.stack([l.float() for l in lses])  # [n, H, Q]
    if sink is not None:
        sl = sink.float()[None, :, None].expand(1, L.shape[1], L.shape[2])
        Lall = torch.cat([L, sl], 0)
    else:
        Lall = L
    m = Lall.amax(0)
    m = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
    w = torch.exp(L - m)  # [n,H,Q]
    denom = torch.exp(Lall - m).sum(0)
    acc = sum(o.float() * (wi / denom).transpose(0, 1)[..., None] for o, wi in zip(outs, w))
    return acc.to(outs[0].dtype)


def mla_decode(q: torch.Tensor, cache: torch.Tensor, block_tables: torch.Tensor, seq_lens: torch.Tensor,
               scale: float, v_dim: int = 512) -> torch.Tensor:
    """Multi-head latent attention for one new token per sequence (absorbed form, fp32): the
    paged cache [num_blocks, block_size, d_qk] holds one latent row per token shared by every
    head; s = scale * q . c, p = softmax over the sequence's tokens, o = p . c[:, :v_dim].
    q [B, Hq, d_qk] -> o [B, Hq, v_dim] in q's dtype."""
    B, Hq, _ = q.shape
    bs = cache.shape[1]
    out = torch.zeros(B, Hq, v_dim, dtype=torch.float32, device=q.device)
    for b in range(B):
        L = int(seq_lens[b])
        if L <= 0:
            continue
        nblk = -(-L // bs)
        rows = cache[block_tables[b, :nblk].long()].reshape(nblk * bs, -1)[:L].float()
        s = (q[b].float() @ rows.t()) * scale
        p = torch.softmax(s, dim=-1)
        out[b] = p @ rows[:, :v_dim]
    return out.to(q.dtype)
