"""dtype names and properties (``utils/dtype_utils.py`` of the Trainium plugin)."""

from __future__ import annotations

import torch

_NAMES = {
    "auto": torch.bfloat16, "bfloat16": torch.bfloat16, "bf16": torch.bfloat16,
    "float16": torch.float16, "fp16": torch.float16, "half": torch.float16,
    "float32": torch.float32, "fp32": torch.float32, "float": torch.float32,
    "fp8": torch.float8_e4m3fn, "fp8_e4m3": torch.float8_e4m3fn, "float8_e4m3fn": torch.float8_e4m3fn,
    "fp8_e5m2": torch.float8_e5m2, "uint8": torch.uint8, "int32": torch.int32, "int64": torch.int64,
}


def to_torch_dtype(x) -> torch.dtype:
    if isinstance(x, torch.dtype):
        return x
    key = str(x).lower().replace("torch.", "")
    if key not in _NAMES:
        raise ValueError(f"unknown dtype {x!r}; known: {sorted(_NAMES)}")
    return _NAMES[key]


def dtype_name(dt: torch.dtype) -> str:
    return str(dt).replace("torch.", "")


def element_size(dt) -> int:
    return torch.empty(0, dtype=to_torch_dtype(dt)).element_size()


def max_finite(dt) -> float:
    dt = to_torch_dtype(dt)
    return float(torch.finfo(dt).max) if dt.is_floating_point else float(torch.iinfo(dt).max)


def mantissa_bits(dt) -> int:
    return {torch.float32: 23, torch.bfloat16: 7, torch.float16: 10, torch.float8_e4m3fn: 3,
            torch.float8_e5m2: 2}[to_torch_dtype(dt)]


def ulp(value: float, dt) -> float:
    """Spacing of representable numbers of ``dt`` near ``value``."""
    import math

    if value == 0:
        return float(torch.finfo(to_torch_dtype(dt)).tiny)
    return 2.0 ** (math.floor(math.log2(abs(value))) - mantissa_bits(dt))
