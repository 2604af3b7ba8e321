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
    # sliding-window KV group (hybrid KV cache): block tables / slot mapping of the windowed
    # layers, whose blocks behind the window have been returned; None when the windowed
    # layers share the full-attention tables
    block_tables_swa: torch.Tensor | None = None
    slot_mapping_swa: torch.Tensor | None = None
    # mixed steps: the first num_decode_seqs sequences are single-token decodes (their query
    # rows are rows 0 .. num_decode_seqs - 1), the rest prompt chunks
    num_decode_seqs: int = 0

    def for_layer(self, window: int | None) -> "AttentionMetadata":
        """The metadata a layer reads: the sliding-window group's tables for a windowed
        layer when the KV cache keeps the two groups apart."""
        if window and self.block_tables_swa is not None:
            import dataclasses

            return dataclasses.replace(self, block_tables=self.block_tables_swa, slot_mapping=self.slot_mapping_swa,
                                       block_tables_swa=None, slot_mapping_swa=None)
        return self


class B200AttentionBackend:
    """Stateless description of the paged-attention backend (the reference's
    ``NeuronAttentionBackend``, ``vllm/attention/attn.py:7``): one K and one V cache per
    attention layer in the HND layout ``[num_blocks, kv_heads, block_size, head_size]``
    (the reference stacks them as ``(2, ...)``, ``attn.py:27-35``), read by
    ``csrc/attention.cu`` through block tables.  Block sizes are powers of two (the kernels
    address blocks with shifts); head sizes are the ones the kernels are built for."""

    name = "B200_PAGED"
    supported_head_sizes = (64, 128, 256)

    @staticmethod
    def get_name() -> str:
        return B200AttentionBackend.name

    @staticmethod
    def get_metadata_cls() -> type:
        return AttentionMetadata

    @staticmethod
    def get_kv_cache_shape(num_blocks: int, block_size: int, num_kv_heads: int, head_size: int) -> tuple:
        return (2, num_blocks, num_kv_heads, block_size, head_size)

    @staticmethod
    def get_supported_head_sizes() -> tuple:
        return B200AttentionBackend.supported_head_sizes

    @staticmethod
    def validate(block_size: int, head_size: int) -> None:
        if block_size <= 0 or block_size & (block_size - 1):
            raise ValueError(f"block_size must be a power of two, got {block_size}")
        if head_size not in B200AttentionBackend.supported_head_sizes:
            raise ValueError(f"head size {head_size} not in {B200AttentionBackend.supported_head_sizes}")
