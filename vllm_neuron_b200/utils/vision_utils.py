"""Vision-encoder batching helpers (``utils/vision_block_packing.py`` / ``vision_utils.py`` of the
Trainium plugin).

``pack_sequences(lengths, block_size)``: first-fit-decreasing packing of per-image patch
sequences into blocks of at most ``block_size`` patches (an image longer than a block gets
blocks of its own).  The vision tower runs one varlen attention call over a packed block, so
fewer, fuller blocks mean fewer launches and less padding.
"""

from __future__ import annotations


def pack_sequences(lengths: list[int], block_size: int) -> list[list[int]]:
    """Returns blocks as lists of sequence indices (each block's total <= block_size, except
    a single sequence longer than a block)."""
    order = sorted(range(len(lengths)), key=lambda i: -lengths[i])
    blocks: list[list[int]] = []
    room: list[int] = []
    for i in order:
        n = lengths[i]
        if n >= block_size:
            blocks.append([i])
            room.append(0)
            continue
        for b, r in enumerate(room):
            if r >= n:
                blocks[b].append(i)
                room[b] -= n
                break
        else:
            blocks.append([i])
            room.append(block_size - n)
    return blocks


def padding_fraction(lengths: list[int], blocks: list[list[int]], block_size: int) -> float:
    used = sum(lengths)
    cap = sum(max(block_size, sum(lengths[i] for i in b)) for b in blocks)
    return 1.0 - used / cap if cap else 0.0
