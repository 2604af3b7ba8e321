"""Shared model plumbing: KV spec, head sharding, weight initialisation."""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn


@dataclass
class LayerSpec:
    """Per-layer KV geometry (``vllm_neuron/model/kv_cache.py:8``)."""

    num_kv_heads: int  # local to this rank
    head_dim: int
    dtype: torch.dtype
    sliding_window: int | None = None
    kind: str = "attention"  # attention | linear_attention (no paged KV)


@dataclass
class KVSpec:
    layers: list[LayerSpec]

    def bytes_per_block(self, block_size: int, windowed: bool | None = None) -> int:
        """KV bytes one block holds across the attention layers (``windowed``: only the
        sliding-window layers / only the others; None: all)."""
        tot = 0
        for l in self.layers:
            if l.kind != "attention":
                continue
            if windowed is not None and bool(l.sliding_window) != windowed:
                continue
            tot += 2 * block_size * l.num_kv_heads * l.head_dim * torch.empty(0, dtype=l.dtype).element_size()
        return tot

    @property
    def sliding_window(self) -> int | None:
        """The window of the sliding-window layers when the model mixes them with
        full-attention layers (one window), else None."""
        att = [l for l in self.layers if l.kind == "attention"]
        wins = {l.sliding_window for l in att if l.sliding_window}
        if len(wins) == 1 and any(not l.sliding_window for l in att):
            return wins.pop()
        return None


def component(ps, name: str) -> dict:
    """Constructor kwargs ``group`` / ``dp_group`` of an embedding or LM head under
    component DP (the TP group and no DP gather unless the component's DP degree is > 1)."""
    g, dp_g = ps.component(name)
    return {"group": g, "dp_group": dp_g}


def kv_head_sharding(num_kv_heads: int, tp: int, tp_rank: int) -> tuple[int, int]:
    """(first kv head, number of kv heads) held by ``tp_rank``.  When TP exceeds
    the KV head count, KV heads are replicated (``model_mxfp4.py:306-313``)."""
    if num_kv_heads >= tp:
        if num_kv_heads % tp:
            raise ValueError(f"kv heads {num_kv_heads} not divisible by tp {tp}")
        n = num_kv_heads // tp
        return tp_rank * n, n
    if tp % num_kv_heads:
        raise ValueError(f"tp {tp} not divisible by kv heads {num_kv_heads}")
    return tp_rank // (tp // num_kv_heads), 1


@torch.no_grad()
def random_init_(module: nn.Module, seed: int = 0, std: float = 0.02) -> None:
    """Deterministic random init for the dummy load format: normal(0, std) for float
    params (norm weights get 1), random MXFP4 codes with scales giving ~std for
    packed expert weights, zeros for biases."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    for name, p in module.named_parameters():
        dev = p.device
        if p.dtype == torch.uint8:
            if name.endswith("_scales") or name.endswith(".s13") or name.endswith(".s2"):
                # e2m1 codes have RMS ~2.93; 2^(120-127) * 2.93 ~= 0.023
                p.data.fill_(120)
            else:
                _fill_chunked(p, lambda n: torch.randint(0, 256, (n,), generator=g, dtype=torch.int32).to(torch.uint8))
            continue
        if "norm" in name and name.endswith("weight"):
            p.data.fill_(1.0)
        elif name.endswith("bias"):
            p.data.zero_()
        elif name.endswith("weight_scale") or name.endswith("input_scale"):  # FP8 dequantisation scales
            p.data.fill_(1.0 if name.endswith("weight_scale") else 0.05)
        else:
            _fill_chunked(p, lambda n: torch.randn(n, generator=g, dtype=torch.float32) * std)


def _fill_chunked(p: torch.Tensor, make, chunk: int = 1 << 26) -> None:
    flat = p.data.view(-1)
    n = flat.numel()
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        flat[s:e].copy_(make(e - s).to(flat.dtype))


@torch.no_grad()
def random_init_device_(module: nn.Module, seed: int = 0, std: float = 0.02) -> None:
    """Same distribution as :func:`random_init_`, generated on the parameter's device
    (fast for multi-GB GPU models; values differ from the CPU generator)."""
    for i, (name, p) in enumerate(module.named_parameters()):
        g = torch.Generator(device=p.device).manual_seed(seed * 1000003 + i)
        if p.dtype == torch.uint8:
            if name.endswith("_scales") or name.endswith(".s13") or name.endswith(".s2"):
                p.data.fill_(120)
            else:
                p.data.copy_(torch.randint(0, 256, p.shape, generator=g, device=p.device, dtype=torch.uint8))
            continue
        if "norm" in name and name.endswith("weight"):
            p.data.fill_(1.0)
        elif name.endswith("bias"):
            p.data.zero_()
        elif name.endswith("weight_scale") or name.endswith("input_scale"):
            p.data.fill_(1.0 if name.endswith("weight_scale") else 0.05)
        elif p.dtype == torch.float8_e4m3fn:
            p.data.copy_(torch.empty(p.shape, device=p.device).normal_(0.0, std, generator=g).to(p.dtype))
        else:
            p.data.normal_(0.0, std, generator=g)
