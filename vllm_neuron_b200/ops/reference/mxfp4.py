"""OCP microscaling (MX) formats.

MXFP4 = e2m1 elements, two per byte (low nibble = even element), one e8m0 scale
(2^(s-127)) per 32 consecutive elements along the contraction dimension.  This is
the HF GPT-OSS checkpoint layout (``*_blocks [.., rows, K/32, 16]`` + ``*_scales
[.., rows, K/32]``; the Trainium plugin dequantises it in
``model/gpt_oss/weight_loaders_bf16.py:264``) and, unchanged, the operand format of
the Blackwell block-scaled tensor-core MMA, so the B200 path keeps it packed.

MXFP8 (e4m3 + e8m0 per 32) is the activation format of the MoE GEMM; the scale is
chosen as in the OCP MX v1.0 spec: X = 2^(floor(log2(amax)) - emax_elem).
"""

from __future__ import annotations

import torch

FP4_VALUES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0)
E4M3_MAX = 448.0
E4M3_EMAX = 8
E2M1_EMAX = 2


def dequant_mxfp4(blocks: torch.Tensor, scales: torch.Tensor, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """blocks [..., K/2] uint8 (or [..., K/32, 16]), scales [..., K/32] uint8 -> [..., K]."""
    if blocks.dim() == scales.dim() + 1:
        blocks = blocks.reshape(*blocks.shape[:-2], -1)
    lut = torch.tensor(FP4_VALUES, dtype=torch.float32, device=blocks.device)
    lo = lut[(blocks & 0x0F).long()]
    hi = lut[(blocks >> 4).long()]
    vals = torch.stack([lo, hi], dim=-1).reshape(*blocks.shape[:-1], blocks.shape[-1] * 2)
    exp = scales.to(torch.int32) - 127
    vals = vals.reshape(*vals.shape[:-1], -1, 32) * torch.pow(2.0, exp.float())[..., None]
    return vals.reshape(*blocks.shape[:-1], -1).to(dtype)


def _e2m1_code(x: torch.Tensor) -> torch.Tensor:
    """Round-to-nearest-even onto the e2m1 grid, return the 4-bit code."""
    mags = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], device=x.device)
    a = x.abs().clamp(max=6.0)
    idx = (a[..., None] - mags).abs().argmin(-1)
    # ties: argmin picks the lower magnitude; fix ties to even code
    lower = mags[idx]
    nxt = mags[(idx + 1).clamp(max=7)]
    tie = ((a - lower) == (nxt - a)) & (idx < 7) & (idx % 2 == 1)
    idx = torch.where(tie, idx + 1, idx)
    sign = (x < 0) & (idx > 0)
    return (idx + sign.long() * 8).to(torch.uint8)


def quantize_mxfp4(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """w [..., K] (K % 32 == 0) -> (blocks [..., K/2] uint8, scales [..., K/32] uint8)."""
    K = w.shape[-1]
    assert K % 32 == 0
    g = w.float().reshape(*w.shape[:-1], K // 32, 32)
    amax = g.abs().amax(-1)
    e = torch.where(amax > 0, torch.floor(torch.log2(amax.clamp_min(1e-38))) - E2M1_EMAX, torch.zeros_like(amax))
    e = e.clamp(-127, 127)
    q = g / torch.pow(2.0, e)[..., None]
    codes = _e2m1_code(q).reshape(*w.shape[:-1], K)
    packed = (codes[..., 0::2] | (codes[..., 1::2] << 4)).to(torch.uint8)
    return packed, (e + 127).to(torch.uint8)


def quantize_mxfp8(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """x [..., K] -> (e4m3 [..., K], e8m0 scales [..., K/32] uint8)."""
    K = x.shape[-1]
    assert K % 32 == 0
    g = x.float().reshape(*x.shape[:-1], K // 32, 32)
    amax = g.abs().amax(-1)
    e = torch.where(amax > 0, torch.floor(torch.log2(amax.clamp_min(1e-38))) - E4M3_EMAX, torch.zeros_like(amax))
    e = e.clamp(-127, 127)
    q = (g / torch.pow(2.0, e)[..., None]).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
    return q.reshape(*x.shape[:-1], K), (e + 127).to(torch.uint8)


def dequant_mxfp8(q: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    K = q.shape[-1]
    g = q.float().reshape(*q.shape[:-1], K // 32, 32)
    return (g * torch.pow(2.0, scales.float() - 127)[..., None]).reshape(*q.shape[:-1], K)
