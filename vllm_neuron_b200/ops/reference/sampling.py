"""Sampling references.

Order of operations as in the Trainium plugin's on-device sampler
(``functional/sampling.py:21``): temperature -> top-k (bounded by ``max_top_k``) ->
softmax -> top-p -> multinomial (or argmax when greedy).  Rejection sampling:
greedy accept-until-first-mismatch plus a bonus token, output ``[B, k+1]`` padded
with -1 (``nn/rejection_sampler.py:12``).
"""

from __future__ import annotations

import torch


def greedy(logits: torch.Tensor) -> torch.Tensor:
    return logits.float().argmax(-1).to(torch.int64)


def topk_topp_filter(logits: torch.Tensor, top_k: torch.Tensor, top_p: torch.Tensor,
                     max_top_k: int = 256) -> tuple[torch.Tensor, torch.Tensor]:
    """Returns (probs over the kept candidates [B, K], candidate ids [B, K]),
    K = min(max_top_k, vocab).  top_k <= 0 means max_top_k."""
    B, V = logits.shape
    K = min(max_top_k, V)
    vals, ids = torch.topk(logits.float(), K, dim=-1)
    k = torch.where(top_k <= 0, torch.full_like(top_k, K), top_k.clamp(max=K))
    ar = torch.arange(K, device=logits.device)[None, :]
    vals = vals.masked_fill(ar >= k[:, None], float("-inf"))
    probs = torch.softmax(vals, dim=-1)
    cdf = probs.cumsum(-1)
    # keep the smallest prefix whose mass reaches top_p (always keep the first)
    keep = (cdf - probs) < top_p[:, None]
    keep[:, 0] = True
    probs = probs * keep
    probs = probs / probs.sum(-1, keepdim=True)
    return probs, ids


def sample(logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor, top_p: torch.Tensor,
           generator: torch.Generator | None = None, max_top_k: int = 256,
           uniform: torch.Tensor | None = None) -> torch.Tensor:
    """Per-row sampling; temperature <= 0 selects greedy for that row.

    ``uniform`` ([B] in [0,1)) makes the draw deterministic: the sampled candidate is
    the first whose CDF exceeds it (inverse-CDF sampling)."""
    greedy_ids = greedy(logits)
    t = temperature.float().clamp_min(1e-6)
    probs, ids = topk_topp_filter(logits.float() / t[:, None], top_k, top_p, max_top_k)
    if uniform is None:
        choice = torch.multinomial(probs, 1, generator=generator).squeeze(-1)
    else:
        cdf = probs.cumsum(-1)
        choice = (cdf <= uniform[:, None].float()).sum(-1).clamp(max=probs.shape[1] - 1)
    sampled = ids.gather(1, choice[:, None]).squeeze(-1)
    return torch.where(temperature <= 0, greedy_ids, sampled)


def rejection_greedy(draft_ids: torch.Tensor, target_ids: torch.Tensor) -> torch.Tensor:
    """draft_ids [B, k]; target_ids [B, k+1] (argmax at each draft position + bonus).
    Output [B, k+1]: target tokens up to and including the first mismatch, -1 after."""
    B, k = draft_ids.shape
    match = (draft_ids == target_ids[:, :k]).int()
    n_acc = match.cumprod(-1).sum(-1)  # accepted drafts
    ar = torch.arange(k + 1, device=draft_ids.device)[None, :]
    return torch.where(ar <= n_acc[:, None], target_ids, torch.full_like(target_ids, -1))


def correct_spec_decode_positions_and_slot_mapping(positions: torch.Tensor, slot_mapping: torch.Tensor,
                                                   num_rejected: torch.Tensor, block_tables: torch.Tensor,
                                                   block_size: int) -> tuple[torch.Tensor, torch.Tensor]:
    """After rejections the next step's positions move back by the number of rejected
    drafts; recompute the slots from the block table
    (``functional/spec_decode_correction.py:23``).  positions/slot_mapping [B, n]."""
    pos = positions - num_rejected[:, None]
    blk = torch.gather(block_tables.long(), 1, (pos // block_size).clamp_min(0))
    slots = blk * block_size + pos % block_size
    slots = torch.where(pos >= 0, slots, torch.full_like(slots, -1))
    return pos, slots


def argsort_unstable(x: torch.Tensor) -> torch.Tensor:
    return torch.argsort(x, stable=False)


def cumsum(x: torch.Tensor) -> torch.Tensor:
    return torch.cumsum(x.float(), dim=-1).to(x.dtype)
