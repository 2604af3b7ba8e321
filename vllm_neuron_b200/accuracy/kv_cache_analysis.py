"""KV-cache inspection (``accuracy/kv_cache_analysis.py`` of the Trainium plugin).

* ``gather_request_kv(k_cache, v_cache, block_ids, seq_len)``: a request's keys and values
  [seq_len, kv_heads, head_dim] out of the paged cache (HND blocks);
* ``compare_kv(a, b)``: per-head error statistics between two such gathers (e.g. this
  engine vs a reference run, or before / after a KV transfer);
* ``kv_stats(k, v)``: magnitude statistics per head (fp8 KV scale selection).
"""

from __future__ import annotations

import torch


def gather_request_kv(k_cache: torch.Tensor, v_cache: torch.Tensor, block_ids: list[int], seq_len: int,
                      k_scale: float = 1.0, v_scale: float = 1.0) -> tuple[torch.Tensor, torch.Tensor]:
    bs = k_cache.shape[2]
    nb = (seq_len + bs - 1) // bs
    idx = torch.tensor(block_ids[:nb], device=k_cache.device, dtype=torch.long)
    k = k_cache.index_select(0, idx).float() * k_scale  # [nb, H, bs, d]
    v = v_cache.index_select(0, idx).float() * v_scale
    k = k.permute(0, 2, 1, 3).reshape(nb * bs, k.shape[1], k.shape[3])[:seq_len]
    v = v.permute(0, 2, 1, 3).reshape(nb * bs, v.shape[1], v.shape[3])[:seq_len]
    return k, v


def compare_kv(a: torch.Tensor, b: torch.Tensor) -> dict:
    err = (a.float() - b.float()).abs()
    ref = b.float().abs().amax(dim=(0, 2)).clamp_min(1e-12)
    return {"max_abs": err.max().item(), "mean_abs": err.mean().item(),
            "max_rel_per_head": (err.amax(dim=(0, 2)) / ref).tolist(),
            "first_bad_position": int((err.amax(dim=(1, 2)) > 1e-2 * ref.max()).nonzero()[0].item())
            if (err.amax(dim=(1, 2)) > 1e-2 * ref.max()).any() else None}


def kv_stats(k: torch.Tensor, v: torch.Tensor) -> dict:
    return {"k_absmax_per_head": k.abs().amax(dim=(0, 2)).tolist(), "v_absmax_per_head": v.abs().amax(dim=(0, 2)).tolist(),
            "k_rms": k.pow(2).mean().sqrt().item(), "v_rms": v.pow(2).mean().sqrt().item()}
