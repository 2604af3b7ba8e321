"""Helpers that line captured tensors of two runs up before comparing them (the reference's
``accuracy/tensor_alignment_utils.py``: ``align_and_truncate_hidden`` ``:48``, ``slice_token``
``:106``, ``count_real_tokens`` ``:126``, ``align_decode_captures`` ``:135``)."""

from __future__ import annotations

import logging

import torch

logger = logging.getLogger(__name__)


def seq_dim_size(t: torch.Tensor) -> int:
    """Tokens of a [tokens, hidden] or [batch, tokens, hidden] tensor."""
    return t.shape[1] if t.dim() == 3 else (t.shape[0] if t.dim() == 2 else 0)


def slice_token(t: torch.Tensor, i: int) -> torch.Tensor:
    """Token ``i`` (keeping the token dimension)."""
    return t[:, i:i + 1] if t.dim() == 3 else t[i:i + 1]


def count_real_tokens(positions: list[int]) -> int:
    """Rows of a padded step that are real tokens: padding repeats the last real position,
    so real rows are the ones whose position rises."""
    return sum(1 for i, p in enumerate(positions) if i == 0 or p > positions[i - 1])


def align_and_truncate_hidden(*tensors: torch.Tensor) -> tuple[list[torch.Tensor], bool]:
    """fp32 copies with a leading batch of one dropped and the hidden dimension cut to the
    smallest one (a padded hidden size on one side); also whether the shapes now agree."""
    ts = [t.float() for t in tensors]
    if max(t.dim() for t in ts) == 3:
        ts = [t[None] if t.dim() == 2 else t for t in ts]
    h = min(t.shape[-1] for t in ts)
    ts = [t[..., :h] for t in ts]
    ts = [t[0] if t.dim() == 3 and t.shape[0] == 1 else t for t in ts]
    return ts, all(t.shape == ts[0].shape for t in ts)


def align_decode_captures(ref: list, target: list) -> list:
    """The reference passes to compare against ``target``: all prefill passes, then the decode
    passes ordered by their largest position, keeping only positions the target also decoded
    (the two runs may have decoded a different number of steps)."""
    pre = [c for c in ref if c.is_prefill]
    rd = sorted((c for c in ref if not c.is_prefill), key=lambda c: max(c.metadata.positions))
    td = [c for c in target if not c.is_prefill]
    if not rd or not td:
        return pre + rd
    have = {max(c.metadata.positions) for c in td}
    dropped = sorted({max(c.metadata.positions) for c in rd} - have)
    if dropped:
        logger.warning("dropping %d reference decode pass(es) without a target pass: %s", len(dropped), dropped)
    return pre + [c for c in rd if max(c.metadata.positions) in have]


def match_passes(ref: list, target: list) -> list[tuple]:
    """(reference pass, target pass) pairs: prefill passes in order, decode passes by their
    largest position."""
    pairs = list(zip([c for c in ref if c.is_prefill], [c for c in target if c.is_prefill]))
    by_pos = {max(c.metadata.positions): c for c in target if not c.is_prefill}
    for c in align_decode_captures(ref, target):
        if not c.is_prefill and max(c.metadata.positions) in by_pos:
            pairs.append((c, by_pos[max(c.metadata.positions)]))
    return pairs
