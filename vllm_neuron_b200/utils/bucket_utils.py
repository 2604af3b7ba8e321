"""Shape-bucket policy.

Decode batches are padded to ``num_seqs_buckets`` (each bucket is one captured CUDA
graph); prefill segments are padded to ``num_batched_tokens_buckets``.  Defaults
and validation follow the Trainium plugin's policy (``vllm_neuron/utils/bucket_utils.py:22-553``):
powers of two from 128 tokens / 1 sequence, always ending at the configured max,
and segmented prefill whenever ``max_num_batched_tokens < max_model_len``.
"""

from __future__ import annotations

import bisect
from dataclasses import dataclass

SUPPORTED_KV_SEGMENT_SIZES = (512, 1024, 2048, 4096, 8192)
MAX_MODEL_LEN_SINGLE_SHOT = 16 * 1024


def next_power_of_2(n: int) -> int:
    return 1 if n <= 1 else 1 << (n - 1).bit_length()


def _pow2_ladder(start: int, last: int) -> list[int]:
    out, b = [], start
    while b < last:
        out.append(b)
        b *= 2
    out.append(last)
    return out


def get_default_num_batched_tokens_buckets(max_num_batched_tokens: int) -> list[int]:
    return _pow2_ladder(128, max_num_batched_tokens)


def get_default_num_seqs_buckets(max_num_seqs: int) -> list[int]:
    return _pow2_ladder(1, max_num_seqs)


def get_default_num_vision_tokens_buckets(max_bucket: int, block: int) -> list[int]:
    return _pow2_ladder(block, max_bucket)


def validate_buckets(name: str, buckets: list[int] | None, maximum: int) -> list[int]:
    if buckets is None:
        raise ValueError(f"{name}: buckets must be provided")
    if not isinstance(buckets, (list, tuple)) or not buckets:
        raise ValueError(f"{name}: must be a non-empty list, got {buckets!r}")
    if any((not isinstance(b, int)) or b < 1 for b in buckets):
        raise ValueError(f"{name}: every bucket must be a positive int, got {buckets!r}")
    out = sorted(set(buckets))
    if out[-1] > maximum:
        raise ValueError(f"{name}: largest bucket {out[-1]} exceeds the maximum {maximum}")
    if out[-1] != maximum:
        out.append(maximum)
    return out


def get_bucket_for_count(count: int, buckets: list[int]) -> int:
    """Smallest bucket >= count (``bucket_utils.py:448``)."""
    i = bisect.bisect_left(buckets, count)
    if i == len(buckets):
        raise ValueError(f"count {count} exceeds the largest bucket {buckets[-1]}")
    return buckets[i]


def get_decode_padded_batch_size(num_reqs: int, buckets: list[int]) -> int:
    return get_bucket_for_count(num_reqs, buckets)


@dataclass
class SegmentedPrefillConfig:
    enabled: bool
    segment_size: int


def resolve_segmented_prefill_config(max_num_batched_tokens: int, max_model_len: int,
                                     kv_segment_size_buckets: list[int] | None = None) -> SegmentedPrefillConfig:
    """Segmented (chunked) prefill is on when one step cannot hold a whole prompt
    (``bucket_utils.py:223-275``).  The segment size is the largest supported size
    not above the token budget."""
    if max_num_batched_tokens >= max_model_len and max_model_len <= MAX_MODEL_LEN_SINGLE_SHOT:
        return SegmentedPrefillConfig(False, max_num_batched_tokens)
    cands = kv_segment_size_buckets or list(SUPPORTED_KV_SEGMENT_SIZES)
    for c in cands:
        if c not in SUPPORTED_KV_SEGMENT_SIZES:
            raise ValueError(f"kv_segment_size {c} not in {SUPPORTED_KV_SEGMENT_SIZES}")
    fit = [c for c in cands if c <= max_num_batched_tokens]
    seg = max(fit) if fit else min(cands)
    return SegmentedPrefillConfig(True, seg)
