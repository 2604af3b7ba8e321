"""Tensor helpers of speculative decoding (the reference's ``utils/spec_decode_utils.py``:
``extract_next_token_ids`` ``:13``, ``compute_token_indices_to_sample`` ``:62``,
``replicate_per_seq_rows`` ``:98``).  All stay on the device (no host synchronisation), so they
can sit inside a captured verify step."""

from __future__ import annotations

import torch


def extract_next_token_ids(sampled: torch.Tensor | list[list[int]], vocab_size: int
                           ) -> tuple[torch.Tensor, torch.Tensor]:
    """Per request: the last accepted token and the number of accepted tokens.  ``sampled`` is
    [requests, k + 1] with -1 after the first rejection (or one list of tokens per request);
    ids outside [0, vocab_size) count as rejected.  Returns two int32 tensors [requests]."""
    if not isinstance(sampled, torch.Tensor):
        width = max((len(x) for x in sampled), default=1)
        sampled = torch.tensor([list(x) + [-1] * (width - len(x)) for x in sampled] or [[-1]], dtype=torch.long)
    if sampled.dim() == 1:
        sampled = sampled[:, None]
    ok = (sampled >= 0) & (sampled < vocab_size)
    # accepted tokens form a prefix: count up to the first invalid entry
    count = ok.to(torch.int32).cumprod(1).sum(1).to(torch.int32)
    last = sampled.gather(1, (count - 1).clamp(min=0).long()[:, None]).squeeze(1).to(torch.int32)
    return last, count


def compute_token_indices_to_sample(last_token_indices: torch.Tensor, num_draft_tokens: torch.Tensor | None,
                                    accepted: torch.Tensor) -> torch.Tensor:
    """Row of each request's last accepted token in the verify batch: the last row of the
    request minus its rejected drafts (``num_draft_tokens + 1 - accepted`` for requests that
    had drafts; unchanged without speculation)."""
    if num_draft_tokens is None:
        return last_token_indices
    nd = num_draft_tokens.to(last_token_indices.device).long()
    rejected = torch.where(nd > 0, nd + 1 - accepted.to(nd.device).long(), torch.zeros_like(nd))
    return last_token_indices - rejected


def replicate_per_seq_rows(per_seq: torch.Tensor, num_repeats: int) -> torch.Tensor:
    """Row i * num_repeats + j = row i (one copy of a per-sequence tensor per verify row)."""
    if num_repeats < 1:
        raise ValueError("num_repeats must be >= 1")
    if num_repeats == 1:
        return per_seq
    idx = torch.arange(per_seq.shape[0] * num_repeats, device=per_seq.device) // num_repeats
    return per_seq.index_select(0, idx)
