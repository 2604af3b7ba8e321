"""Per-step attention metadata built by the model runner and read by every attention layer."""

from __future__ import annotations

from dataclasses import dataclass, field

import torch


@dataclass
class AttentionMetadata:
    """All tensors live on the model's device.

    ``query_start_loc`` [B+1] and ``seq_lens`` [B] (keys in the cache after this
    step's tokens are written) are int32; ``block_tables`` [B, max_blocks] int32;
    ``slot_mapping`` [T] int64 with -1 for padding tokens.  ``is_decode`` means
    every sequence contributes exactly one query token.  ``max_query_len`` /
    ``max_seq_len`` are host ints (upper bounds, used for launch sizing).
    ``logits_indices`` [B] selects, per sequence, the flat token whose hidden state
    is sampled.
    """

    num_tokens: int
    num_seqs: int
    is_decode: bool
    query_start_loc: torch.Tensor
    seq_lens: torch.Tensor
    block_tables: torch.Tensor
    slot_mapping: torch.Tensor
    logits_indices: torch.Tensor
    max_query_len: int
    max_seq_len: int
    # scratch for split-KV decode (allocated once per runner, reused by every layer)
    workspace: torch.Tensor | None = None
    num_splits: int = 1
    extras: dict = field(default_factory=dict)
    # decode context parallelism: the DCP group (ranks that hold the same KV heads and
    # split the tokens of every sequence block by block); None without DCP
    cp_group: object = None
