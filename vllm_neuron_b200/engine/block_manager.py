"""Paged KV-cache block manager with prefix caching.

Blocks of ``block_size`` token slots are handed out from a free queue.  With prefix
caching, a block whose ``block_size`` tokens are all computed is registered under
a chained content hash (parent hash, token ids, extra keys such as image hashes);
a later request whose prompt starts with the same blocks shares them (reference
counted) and skips their prefill.  Freed blocks keep their hash and stay reusable
until the free queue hands them out again (LRU order: blocks are appended at the
tail when freed and taken from the head).

Block 0 is reserved as the null block: padded decode rows point at it and never
write to it.  This is the role vLLM's KV block manager plays for the Trainium
plugin (which keeps vLLM's manager, ``docs/design/vllm/prefix-caching.md``).
"""

from __future__ import annotations

import hashlib
import struct
from collections import OrderedDict

from .request import Request


def hash_block(parent: bytes | None, tokens: tuple[int, ...], extra: tuple = ()) -> bytes:
    h = hashlib.sha256()
    h.update(parent or b"root")
    h.update(struct.pack(f"<{len(tokens)}q", *tokens))
    if extra:
        h.update(repr(extra).encode())
    return h.digest()


class BlockPool:
    def __init__(self, num_blocks: int, enable_caching: bool):
        if num_blocks < 2:
            raise ValueError("need at least 2 KV blocks")
        self.num_blocks = num_blocks
        self.enable_caching = enable_caching
        self.ref_cnt = [0] * num_blocks
        self.block_hash: list[bytes | None] = [None] * num_blocks
        self.cached: dict[bytes, int] = {}
        # free queue: OrderedDict used as an LRU (head = next to hand out)
        self.free: OrderedDict[int, None] = OrderedDict((b, None) for b in range(1, num_blocks))
        self.ref_cnt[0] = 1 << 30  # null block never freed

    @property
    def num_free(self) -> int:
        return len(self.free)

    def usage(self) -> float:
        return 1.0 - self.num_free / (self.num_blocks - 1)

    def allocate(self, n: int) -> list[int]:
        if n > len(self.free):
            raise MemoryError(f"need {n} KV blocks, {len(self.free)} free")
        out = []
        for _ in range(n):
            b, _ = self.free.popitem(last=False)
            h = self.block_hash[b]
            if h is not None:
                if self.cached.get(h) == b:
                    del self.cached[h]
                self.block_hash[b] = None
            self.ref_cnt[b] = 1
            out.append(b)
        return out

    def touch(self, b: int) -> None:
        """Take a reference on a cached block (removing it from the free queue)."""
        if self.ref_cnt[b] == 0:
            self.free.pop(b, None)
        self.ref_cnt[b] += 1

    def free_blocks(self, blocks: list[int]) -> None:
        # free in reverse so the tail of a sequence is evicted first
        for b in reversed(blocks):
            if b == 0:
                continue
            self.ref_cnt[b] -= 1
            if self.ref_cnt[b] < 0:
                raise RuntimeError(f"double free of KV block {b}")
            if self.ref_cnt[b] == 0:
                if self.enable_caching and self.block_hash[b] is not None:
                    self.free[b] = None  # reusable, evicted last
                else:
                    # holds nothing reusable: hand it out before any cached block
                    self.block_hash[b] = None
                    self.free[b] = None
                    self.free.move_to_end(b, last=False)

    def register(self, b: int, h: bytes) -> None:
        if not self.enable_caching:
            return
        if self.block_hash[b] is None and h not in self.cached:
            self.block_hash[b] = h
            self.cached[h] = b

    def lookup(self, h: bytes) -> int | None:
        return self.cached.get(h) if self.enable_caching else None


class KVCacheManager:
    """Blocks of the full-attention layers (``pool``) and, for models that mix sliding-window
    and full-attention layers, a second group for the windowed layers (``swa_pool``, the
    reference's hybrid KV-cache groups, ``neuron_model_runner.py:3787,3966-3986``).  A
    request's windowed-layer table keeps one entry per logical block; before a step, the
    entries wholly behind the window of its first query (keys j > p - W stay visible to
    query p) are returned to the pool and become the null block, so a windowed layer holds
    about W / block_size + 1 blocks per sequence instead of the whole context.  Kernels read
    no block before the window.  Prefix caching applies to the full-attention group only,
    and is off whenever the windowed group is kept apart."""

    def __init__(self, num_blocks: int, block_size: int, enable_caching: bool = False,
                 sliding_window: int | None = None, swa_blocks: int = 0):
        self.block_size = block_size
        self.pool = BlockPool(num_blocks, enable_caching)
        self.enable_caching = enable_caching
        self._hashes: dict[str, list[bytes]] = {}
        self._registered: dict[str, int] = {}  # leading blocks already registered per request
        self.window = sliding_window if swa_blocks else None
        self.swa_pool = BlockPool(swa_blocks, False) if swa_blocks else None
        if self.swa_pool is not None and enable_caching:
            raise ValueError("prefix caching with a separate sliding-window KV group is not supported")

    # -------------------------------------------------------------- prefix cache
    def _block_hashes(self, req: Request, upto_tokens: int) -> list[bytes]:
        hs = self._hashes.setdefault(req.request_id, [])
        toks = req.all_token_ids
        bs = self.block_size
        extra = tuple(getattr(req, "mm_hashes", ()) or ())
        while (len(hs) + 1) * bs <= upto_tokens:
            i = len(hs)
            hs.append(hash_block(hs[-1] if hs else None, tuple(toks[i * bs:(i + 1) * bs]), extra))
        return hs

    def get_computed_blocks(self, req: Request) -> tuple[list[int], int]:
        """Longest cached prefix of full blocks; never the whole prompt (the last
        prompt token is always recomputed to produce logits)."""
        if not self.enable_caching:
            return [], 0
        hs = self._block_hashes(req, req.num_prompt_tokens)
        blocks = []
        for h in hs:
            b = self.pool.lookup(h)
            if b is None:
                break
            blocks.append(b)
        while blocks and len(blocks) * self.block_size >= req.num_prompt_tokens:
            blocks.pop()
        return blocks, len(blocks) * self.block_size

    # -------------------------------------------------------------- allocation
    def blocks_needed(self, req: Request, num_new_tokens: int, num_cached_blocks: int = 0) -> int:
        total = req.num_computed_tokens + num_new_tokens
        have = len(req.block_ids) + num_cached_blocks
        need = -(-total // self.block_size)
        return max(0, need - have)

    def can_allocate(self, n: int, watermark: int = 0) -> bool:
        return self.pool.num_free - n >= watermark

    def _trim_window(self, req: Request) -> None:
        """Return the windowed-layer blocks no query from ``num_computed_tokens`` on can see."""
        first_key = req.num_computed_tokens - self.window + 1
        n_dead = max(0, first_key) // self.block_size
        n_dead = min(n_dead, len(req.swa_block_ids))
        if n_dead > req.swa_freed:
            dead = req.swa_block_ids[req.swa_freed:n_dead]
            self.swa_pool.free_blocks(dead)
            req.swa_block_ids[req.swa_freed:n_dead] = [0] * (n_dead - req.swa_freed)
            req.swa_freed = n_dead

    def allocate_slots(self, req: Request, num_new_tokens: int, computed_blocks: list[int] | None = None) -> bool:
        total = req.num_computed_tokens + num_new_tokens
        if self.swa_pool is not None:
            self._trim_window(req)
            n_swa = max(0, -(-total // self.block_size) - len(req.swa_block_ids))
            if n_swa > self.swa_pool.num_free:
                return False
        else:
            n_swa = 0
        if not computed_blocks and total <= len(req.block_ids) * self.block_size:
            return True  # the common decode case: the current block has room
        computed_blocks = computed_blocks or []
        n = self.blocks_needed(req, num_new_tokens, len(computed_blocks))
        # cached blocks taken from the free queue reduce the free count too
        n_cached_free = sum(1 for b in computed_blocks if self.pool.ref_cnt[b] == 0)
        if n + n_cached_free > self.pool.num_free:
            return False
        for b in computed_blocks:
            self.pool.touch(b)
        req.block_ids.extend(computed_blocks)
        req.block_ids.extend(self.pool.allocate(n))
        if n_swa:
            req.swa_block_ids.extend(self.swa_pool.allocate(n_swa))
        return True

    def cache_full_blocks(self, req: Request) -> None:
        """Register blocks that became full after this step's tokens were computed."""
        if not self.enable_caching:
            return
        n_full = min(min(req.num_computed_tokens, req.num_tokens) // self.block_size, len(req.block_ids))
        done = self._registered.get(req.request_id, 0)
        if n_full <= done:
            return
        hs = self._block_hashes(req, n_full * self.block_size)
        for i in range(done, n_full):
            self.pool.register(req.block_ids[i], hs[i])
        self._registered[req.request_id] = n_full

    def free(self, req: Request) -> None:
        self.pool.free_blocks(req.block_ids)
        req.block_ids = []
        if self.swa_pool is not None:
            self.swa_pool.free_blocks(req.swa_block_ids)  # null entries are skipped
            req.swa_block_ids = []
            req.swa_freed = 0
        self._hashes.pop(req.request_id, None)
        self._registered.pop(req.request_id, None)

    @property
    def usage(self) -> float:
        return self.pool.usage()
