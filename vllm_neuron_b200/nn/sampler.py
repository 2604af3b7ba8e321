"""Vocab-parallel on-device sampler.

Each TP rank holds logits for its vocab slice.  As in the Trainium plugin's sampler
(``nn/sampler.py:56-169``, ``functional/topk.py:32-115``, ``functional/argmax.py:26``):
* greedy batches: local argmax per rank, all-gather of (value, index) pairs, global
  argmax (ties resolve to the lowest rank, i.e. the lowest token id);
* otherwise: local top-``max_top_k`` candidates per rank, all-gather, then
  temperature / top-k / top-p / inverse-CDF draw over the merged candidates.
The draw uses a per-row uniform supplied by the host, identical on every rank, so
all ranks produce the same token without a broadcast.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from .. import ops
from ..parallel.state import GroupCoordinator


class Sampler(nn.Module):
    def __init__(self, group: GroupCoordinator, vocab_start: int, vocab_size: int, max_top_k: int = 256,
                 sampling_groups: tuple[GroupCoordinator, GroupCoordinator] | None = None):
        super().__init__()
        self.group = group
        self.vocab_start = vocab_start
        self.vocab_size = vocab_size
        self.max_top_k = max_top_k
        # sampling DP: (all-to-all group of consecutive TP ranks, gather group across them)
        self.sdp = sampling_groups if (sampling_groups and sampling_groups[0].world_size > 1) else None

    def _mask_padding(self, logits: torch.Tensor) -> torch.Tensor:
        # vocab padding rows (when V % tp != 0) must never win
        n_valid = self.vocab_size - self.vocab_start
        if n_valid < logits.shape[1]:
            logits = logits.clone()
            logits[:, max(n_valid, 0):] = float("-inf")
        return logits

    def greedy(self, logits: torch.Tensor) -> torch.Tensor:
        logits = self._mask_padding(logits)
        val, idx = ops.argmax(logits)
        if self.group.world_size == 1:
            return idx
        pair = torch.stack([val, (idx + self.vocab_start).to(torch.float32)], dim=-1)  # [B,2]
        # indices < 2^24 are exact in fp32 (vocab <= 16.7M)
        allp = self.group.all_gather(pair.unsqueeze(0), dim=0)  # [tp,B,2]
        best = allp[..., 0].argmax(0)  # first max = lowest rank
        return allp[..., 1].gather(0, best[None]).squeeze(0).to(torch.int64)

    def forward(self, logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor, top_p: torch.Tensor,
                uniform: torch.Tensor, all_greedy: bool) -> torch.Tensor:
        if all_greedy:
            return self.greedy(logits)
        logits = self._mask_padding(logits)
        if self.group.world_size == 1:
            return ops.sample(logits, temperature, top_k, top_p, uniform, self.max_top_k)
        cand_v, cand_i = self.candidates(logits, masked=True)
        pos = ops.sample(cand_v, temperature, top_k, top_p, uniform, self.max_top_k)
        return cand_i.gather(1, pos[:, None]).squeeze(1).to(torch.int64)

    def candidates(self, logits: torch.Tensor, masked: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
        """Top-``max_top_k`` candidates of every vocab shard, gathered over the TP group:
        (logits [B, tp*K] fp32, global vocab ids [B, tp*K] int64).  Any top-k / top-p
        selection over the full vocabulary is contained in this set."""
        if not masked:
            logits = self._mask_padding(logits)
        if self.sdp is not None:
            return self._candidates_sdp(logits)
        K = min(self.max_top_k, logits.shape[1])
        vals, ids = torch.topk(logits.float(), K, dim=-1)
        ids = ids + self.vocab_start
        if self.group.world_size == 1:
            return vals, ids.to(torch.int64)
        allv = self.group.all_gather(vals.unsqueeze(0), dim=0)  # [tp,B,K]
        alli = self.group.all_gather(ids.unsqueeze(0), dim=0)
        B = logits.shape[0]
        return allv.permute(1, 0, 2).reshape(B, -1), alli.permute(1, 0, 2).reshape(B, -1).to(torch.int64)

    def _candidates_sdp(self, logits: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Sampling DP (``functional/topk.py:130``, ``sampling.py:106-161``): an all-to-all
        inside each group of ``s`` consecutive TP ranks swaps batch for vocab, so a rank
        holds B/s rows over the s vocab shards of its group; one top-K over that span; the
        candidates are gathered over the ranks holding the other spans and then over the
        row chunks.  The candidate set per row is (tp/s)*K instead of tp*K and contains the
        same global top-K."""
        a2a, gat = self.sdp
        s = a2a.world_size
        B, Vl = logits.shape
        Bp = -(-B // s) * s
        x = logits.float()
        if Bp != B:
            x = torch.cat([x, torch.full((Bp - B, Vl), float("-inf"), device=x.device)], 0)
        span = a2a.all_to_all(x, scatter_dim=0, gather_dim=1)  # [Bp/s, s*Vl]
        K = min(self.max_top_k, span.shape[1])
        vals, ids = torch.topk(span, K, dim=-1)
        ids = ids + (self.vocab_start - a2a.rank_in_group * Vl)  # first vocab id of the group's span
        allv = gat.all_gather(vals.unsqueeze(0), dim=0)  # [tp/s, Bp/s, K]
        alli = gat.all_gather(ids.unsqueeze(0), dim=0)
        rows = Bp // s
        cv = allv.permute(1, 0, 2).reshape(rows, -1)
        ci = alli.permute(1, 0, 2).reshape(rows, -1)
        cv = a2a.all_gather(cv, dim=0)[:B]  # row chunks back in order
        ci = a2a.all_gather(ci, dim=0)[:B]
        return cv, ci.to(torch.int64)
