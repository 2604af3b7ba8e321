"""RMSNorm references (``GptOssRMSNorm``, ``model/gpt_oss/model_mxfp4.py:101``;
``functional/rmsnorm_quant.py:87`` for the fp8 variant)."""

from __future__ import annotations

import torch


def rms_norm(x: torch.Tensor, weight: torch.Tensor | None, eps: float = 1e-5) -> torch.Tensor:
    """y = x * rsqrt(mean(x^2) + eps) * w, computed in fp32, cast back to x.dtype."""
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    if weight is not None:
        y = y * weight.float()
    return y.to(x.dtype)


def fused_add_rms_norm(x: torch.Tensor, residual: torch.Tensor | None, weight: torch.Tensor,
                       eps: float = 1e-5) -> tuple[torch.Tensor, torch.Tensor]:
    """residual' = x + residual; returns (rms_norm(residual'), residual')."""
    r = x if residual is None else (x.float() + residual.float()).to(x.dtype)
    return rms_norm(r, weight, eps), r


def rmsnorm_quant_fp8(x: torch.Tensor, weight: torch.Tensor, eps: float, scale: float,
                      fp8_max: float = 448.0) -> torch.Tensor:
    """RMSNorm then static per-tensor fp8 e4m3 quantisation: q = clamp(y / scale)."""
    y = rms_norm(x.float(), weight, eps)
    return (y / scale).clamp(-fp8_max, fp8_max).to(torch.float8_e4m3fn)
