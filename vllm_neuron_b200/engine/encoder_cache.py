"""On-device cache of vision-encoder outputs (``EncoderCacheBlocks``,
``vllm_neuron/vllm/worker/encoder_cache_blocks.py:59``).

A preallocated ``[num_blocks, block_size, fat_dim]`` buffer holds, per image token, the
merged embedding followed by its deepstack features (``fat_dim = hidden * (1 + n_deep)``).
An image occupies ceil(tokens / block_size) blocks from a free list; prefill chunks that
cover part of an image gather exactly the rows they need, so an image is encoded once
even when its prompt is prefilled in several segments.  Blocks return to the free list
when the request finishes.
"""

from __future__ import annotations

import torch


class EncoderCache:
    def __init__(self, num_blocks: int, block_size: int, fat_dim: int, dtype, device):
        self.block_size = block_size
        self.fat_dim = fat_dim
        self.buf = torch.zeros(num_blocks, block_size, fat_dim, dtype=dtype, device=device)
        self.free = list(range(num_blocks))
        self.items: dict[tuple[str, int], tuple[list[int], int]] = {}

    def has(self, req_id: str, item: int) -> bool:
        return (req_id, item) in self.items

    def put(self, req_id: str, item: int, fat: torch.Tensor) -> None:
        n = fat.shape[0]
        need = -(-n // self.block_size)
        if need > len(self.free):
            raise MemoryError(f"encoder cache full: need {need} blocks, {len(self.free)} free")
        blocks = [self.free.pop() for _ in range(need)]
        flat = self.buf.view(-1, self.fat_dim)
        idx = torch.cat([torch.arange(b * self.block_size, (b + 1) * self.block_size) for b in blocks])[:n]
        flat[idx.to(flat.device)] = fat.to(flat.dtype)
        self.items[(req_id, item)] = (blocks, n)

    def gather(self, req_id: str, item: int, rows: torch.Tensor) -> torch.Tensor:
        blocks, _ = self.items[(req_id, item)]
        bt = torch.tensor(blocks, device=rows.device)
        flat_rows = bt[rows // self.block_size] * self.block_size + rows % self.block_size
        return self.buf.view(-1, self.fat_dim)[flat_rows]

    def release(self, req_id: str) -> None:
        for key in [k for k in self.items if k[0] == req_id]:
            blocks, _ = self.items.pop(key)
            self.free.extend(blocks)

    @property
    def num_free(self) -> int:
        return len(self.free)
