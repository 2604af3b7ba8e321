"""Rotary embeddings.

* YaRN frequencies and attention factor as GPT-OSS uses them
  (``GptOssRotaryEmbedding``, ``model/gpt_oss/model_mxfp4.py:141-197``; concentration
  0.1*ln(factor)+1 multiplies cos/sin).
* Split-half ("neox") rotation: first half / second half of the head dim.
* Interleaved multimodal M-RoPE sections for Qwen3-VL (``model/qwen3_vl/utils/mrope.py``).
"""

from __future__ import annotations

import math

import torch


def yarn_inv_freq(head_dim: int, theta: float, factor: float = 1.0, original_max_pos: int = 4096,
                  beta_fast: float = 32.0, beta_slow: float = 1.0,
                  truncate: bool = False) -> tuple[torch.Tensor, float]:
    """Inverse frequencies and attention scaling of YaRN (Peng et al. 2023, arXiv 2309.00071)."""
    half = head_dim // 2
    pos_freqs = theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim)
    inv_extra = 1.0 / pos_freqs
    if factor == 1.0:
        return inv_extra.float(), 1.0
    inv_inter = 1.0 / (factor * pos_freqs)

    def find_dim(n_rot: float) -> float:
        return (head_dim * math.log(original_max_pos / (n_rot * 2 * math.pi))) / (2 * math.log(theta))

    low = find_dim(beta_fast)
    high = find_dim(beta_slow)
    if truncate:
        low, high = math.floor(low), math.ceil(high)
    low, high = max(low, 0), min(high, head_dim - 1)
    if low == high:
        high += 0.001
    ramp = (torch.arange(half, dtype=torch.float64) - low) / (high - low)
    extra_factor = 1.0 - ramp.clamp(0, 1)
    inv = inv_inter * (1 - extra_factor) + inv_extra * extra_factor
    attn_factor = 0.1 * math.log(factor) + 1.0
    return inv.float(), attn_factor


def llama3_inv_freq(head_dim: int, theta: float, factor: float, low_freq_factor: float, high_freq_factor: float,
                    original_max_pos: int) -> torch.Tensor:
    """Llama 3.x frequency scaling: long wavelengths divided by ``factor``, short ones kept,
    a smooth interpolation in between (Meta's published Llama 3.1 RoPE recipe)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    low_wl = original_max_pos / low_freq_factor
    high_wl = original_max_pos / high_freq_factor
    wl = 2 * math.pi / inv
    scaled = torch.where(wl > low_wl, inv / factor, inv)
    smooth = (original_max_pos / wl - low_freq_factor) / (high_freq_factor - low_freq_factor)
    mid = (1 - smooth) * scaled / factor + smooth * scaled
    is_mid = (wl >= high_wl) & (wl <= low_wl)
    return torch.where(is_mid, mid, scaled).float()


def rope_cos_sin(positions: torch.Tensor, inv_freq: torch.Tensor, attn_factor: float = 1.0,
                 dtype: torch.dtype = torch.float32) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin of shape [T, head_dim/2] (half layout)."""
    freqs = positions.to(torch.float32)[:, None] * inv_freq.to(positions.device, torch.float32)[None, :]
    return (freqs.cos() * attn_factor).to(dtype), (freqs.sin() * attn_factor).to(dtype)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x: [T, heads, d]; cos/sin: [T, d/2].  Rotation of the two halves, in fp32."""
    d2 = x.shape[-1] // 2
    xf = x.float()
    x1, x2 = xf[..., :d2], xf[..., d2:]
    c = cos.float()[:, None, :]
    s = sin.float()[:, None, :]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1).to(x.dtype)


def mrope_cos_sin(positions_3d: torch.Tensor, inv_freq: torch.Tensor, mrope_section: list[int],
                  interleaved: bool = True, dtype: torch.dtype = torch.float32) -> tuple[torch.Tensor, torch.Tensor]:
    """Multimodal RoPE.  positions_3d: [3, T] (temporal, height, width).  Frequency
    slot j takes its position from axis a(j): interleaved layout assigns
    t,h,w,t,h,w,... over the first 3*min(section) slots then t for the rest
    (Qwen3-VL); the non-interleaved layout uses contiguous sections."""
    half = inv_freq.shape[0]
    freqs = positions_3d.to(torch.float32)[:, :, None] * inv_freq.to(positions_3d.device)[None, None, :]  # [3,T,half]
    axis = torch.zeros(half, dtype=torch.long)
    if interleaved:
        for a in (1, 2):
            idx = torch.arange(a, min(mrope_section[a] * 3, half), 3)
            axis[idx] = a
    else:
        off = 0
        for a, n in enumerate(mrope_section):
            axis[off:off + n] = a
            off += n
    sel = freqs.gather(0, axis.to(freqs.device)[None, None, :].expand(1, freqs.shape[1], half)).squeeze(0)
    return sel.cos().to(dtype), sel.sin().to(dtype)
