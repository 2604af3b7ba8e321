"""Decode context parallelism (DCP): the KV cache of every sequence is split across the
ranks of a DCP group, which hold the same KV heads.

Layout: token t of a sequence lives on group rank ``(t // block_size) % dcp`` at local index
``(t // (block_size * dcp)) * block_size + t % block_size`` of the virtual block
``t // (block_size * dcp)`` of the (replicated) block table, so each rank keeps 1/dcp of the
context and the scheduler counts blocks of ``block_size * dcp`` tokens
(``vllm/worker/neuron_model_runner.py:279-328`` deals tokens the same way, interleave size =
block size).

One attention call (decode or chunked prefill) on every rank of the group:

1. all-gather the query heads over the group: every rank now has the queries of all heads
   that read its KV heads;
2. attention of those queries over the rank's own tokens -> normalised partial output and
   LSE, without sinks (``ops.attention_shard``: the paged kernels in shard mode);
3. all-gather the LSEs; the global LSE adds the sink logit once; each partial is scaled by
   ``exp(lse_rank - lse_global)``;
4. reduce-scatter over heads: each rank gets the merged output of its own heads.

The same steps as the reference's decode DCP (``functional/attention/attention_decode.py:
589-592,717-751``); collectives are NCCL (gloo on CPU).  Sliding windows and causal masks
are in global positions inside the kernels.
"""

from __future__ import annotations

import torch

from .. import ops

_sinks_cache: dict[tuple[int, int], torch.Tensor] = {}


def _group_sinks(group, sinks: torch.Tensor) -> torch.Tensor:
    """Sinks of every query head of the group (gathered once per sinks tensor)."""
    key = (id(group), sinks.data_ptr())
    g = _sinks_cache.get(key)
    if g is None:
        g = group.all_gather(sinks.float().contiguous(), dim=0)
        # a gather recorded into a CUDA graph has not run yet: keep it local to that graph
        if not (sinks.is_cuda and torch.cuda.is_current_stream_capturing()):
            _sinks_cache[key] = g
    return g


def merge_partials(o: torch.Tensor, lse: torch.Tensor, lse_all: torch.Tensor,
                   sinks: torch.Tensor | None) -> torch.Tensor:
    """Scale this rank's partial ``o`` [T, H, d] by ``exp(lse - lse_global)``.

    ``lse_all`` [n, T, H] holds every rank's LSE (natural log); ``sinks`` [H] are joined to
    the global denominator once.  Returns fp32; summing the results of all ranks gives the
    exact attention output."""
    parts = lse_all.float()
    if sinks is not None:
        parts = torch.cat([parts, sinks.float().view(1, 1, -1).expand(1, parts.shape[1], -1)], 0)
    lse_g = torch.logsumexp(parts, dim=0)  # -inf where no rank sees a key and there is no sink
    w = torch.exp(lse.float() - lse_g)
    w = torch.nan_to_num(w, nan=0.0)  # (-inf) - (-inf)
    return o.float() * w.unsqueeze(-1)


def dcp_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, meta, scale: float,
                  sinks: torch.Tensor | None, window: int | None, k_scale: float, v_scale: float) -> torch.Tensor:
    """Attention of this rank's query heads q [T, Hl, d] under DCP -> [T, Hl, d]."""
    g = meta.cp_group
    n, r = g.world_size, g.rank_in_group
    qa = g.all_gather(q.contiguous(), dim=1)  # [T, n * Hl, d]
    o, lse = ops.attention_shard(qa, k_cache, v_cache, meta, scale, window, k_scale, v_scale, r, n)
    lse_all = g.all_gather(lse.unsqueeze(0).contiguous(), dim=0)  # [n, T, n * Hl]
    s_all = _group_sinks(g, sinks) if sinks is not None else None
    part = merge_partials(o, lse, lse_all, s_all)
    return g.reduce_scatter(part, dim=1).to(q.dtype)
