"""Synthetic model for disaggregated-inference (KV transfer) testing.

Semantics of the Trainium plugin's test-only ``SyntheticNeuronModel``
(``model/synthetic/synthetic.py:62``, fill / verify in ``sharding.py:149,235``): no weights
and no network.  Every step writes a deterministic value into the paged KV cache for each
(layer, K|V, global kv head, position, dim), and checks that every position before the step
still holds its expected value.  The sampled token reports the outcome:

* ``TOKEN_SUCCESS`` (5)  all earlier positions verified (e.g. after a KV transfer);
* ``TOKEN_FAIL`` (6)     a mismatch was found;
* ``TOKEN_EMPTY`` (7)    nothing to verify (the step starts at position 0).

Values are integers in [1, 251], exact in bf16 / fp16 / fp32, and differ per coordinate, so a
misplaced block, head or position is detected.  Registered only when
``VLLM_B200_SYNTHETIC_MODEL=1``.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn

from .base import KVSpec, LayerSpec, kv_head_sharding

TOKEN_SUCCESS, TOKEN_FAIL, TOKEN_EMPTY = 5, 6, 7


@dataclass
class SyntheticConfig:
    num_hidden_layers: int = 4
    num_key_value_heads: int = 4
    head_dim: int = 64
    vocab_size: int = 32
    max_position_embeddings: int = 4096
    eos_token_id: int | None = None

    @classmethod
    def from_hf(cls, d: dict, quantization: str | None = None) -> "SyntheticConfig":
        keys = cls.__dataclass_fields__
        return cls(**{k: v for k, v in d.items() if k in keys})


def kv_value(layer: int, which: int, head: torch.Tensor, pos: torch.Tensor, dim: torch.Tensor) -> torch.Tensor:
    """Deterministic fill value for broadcastable integer coordinate tensors."""
    return ((layer * 31 + which * 17 + head * 13 + pos * 7 + dim * 3) % 251 + 1).float()


class _Head:
    def __init__(self, start: int):
        self.start = start


class SyntheticModel(nn.Module):
    config_class = SyntheticConfig

    def __init__(self, cfg: SyntheticConfig, ps, dtype=torch.bfloat16, device="cpu", kv_dtype=None):
        super().__init__()
        self.cfg = cfg
        self.dtype = dtype
        self.kv_dtype = kv_dtype or dtype
        tp = ps.tp
        self.h0, self.nkv = kv_head_sharding(cfg.num_key_value_heads, tp.world_size, tp.rank_in_group)
        self.per = -(-cfg.vocab_size // tp.world_size)
        self.lm_head = _Head(tp.rank_in_group * self.per)
        self.layers = nn.ModuleList([nn.Module() for _ in range(cfg.num_hidden_layers)])
        self.register_buffer("_anchor", torch.zeros(1, dtype=dtype, device=device), persistent=False)

    def get_kv_spec(self) -> KVSpec:
        return KVSpec([LayerSpec(self.nkv, self.cfg.head_dim, self.kv_dtype) for _ in self.layers])

    def load_weights(self, weights) -> set:
        return set()

    def forward(self, input_ids, positions, meta, kv_caches, inputs_embeds=None):
        dev = positions.device
        T = positions.shape[0]
        d = self.cfg.head_dim
        heads = torch.arange(self.h0, self.h0 + self.nkv, device=dev)
        dims = torch.arange(d, device=dev)
        pos = positions.long()
        B = meta.num_seqs
        qsl = meta.query_start_loc.long()
        seq_lens = meta.seq_lens.long()
        q_lens = qsl[1:B + 1] - qsl[:B]
        prior = (seq_lens - q_lens).clamp_min(0)  # positions before this step, per sequence
        bt = meta.block_tables.long()
        kc0 = kv_caches[0][0]
        bs = kc0.shape[2]
        L = bt.shape[1] * bs
        p = torch.arange(L, device=dev)
        valid = p[None, :] < prior[:, None]  # [B, L]
        blk = bt.gather(1, (p // bs)[None, :].expand(B, L))
        off = (p % bs)[None, :].expand(B, L)
        bad = torch.zeros(B, dtype=torch.bool, device=dev)
        for i, (kc, vc) in enumerate(kv_caches):
            # verify before writing this step's tokens
            for which, cache in ((0, kc), (1, vc)):
                got = cache[blk, :, off, :].float()  # [B, L, H, d]
                want = kv_value(i, which, heads[None, None, :, None], p[None, :, None, None],
                                dims[None, None, None, :])
                mism = ((got - want).abs() > 0).any(-1).any(-1) & valid
                bad |= mism.any(-1)
            kvals = kv_value(i, 0, heads[None, :, None], pos[:, None, None], dims[None, None, :])
            vvals = kv_value(i, 1, heads[None, :, None], pos[:, None, None], dims[None, None, :])
            # padding rows (slot -1) write the reserved null block 0, which no request reads
            slots = meta.slot_mapping.long().clamp_min(0)
            kc[slots // bs, :, slots % bs] = kvals.to(kc.dtype)
            vc[slots // bs, :, slots % bs] = vvals.to(vc.dtype)
        tok = torch.where(prior > 0, torch.where(bad, TOKEN_FAIL, TOKEN_SUCCESS),
                          torch.full_like(prior, TOKEN_EMPTY))
        # hidden state of every token = its sequence's outcome token
        seq_of = torch.searchsorted(qsl[1:B + 1], torch.arange(T, device=dev), right=True).clamp(max=B - 1)
        return tok[seq_of].to(self._anchor.dtype)[:, None]

    def compute_logits(self, h: torch.Tensor) -> torch.Tensor:
        ids = torch.arange(self.lm_head.start, self.lm_head.start + self.per, device=h.device)
        return torch.where(ids[None, :] == h.long(), 30.0, -30.0).to(torch.float32)
