"""dtype names and properties (``utils/dtype_utils.py`` of the Trainium plugin:
``FP8_CLAMP_MAX`` ``:17-41``, ``kv_cache_dtype_str_to_dtype`` ``:44``).

B200 tensor cores and conversions use the OCP e4m3fn format (no infinities), whose largest
finite value is 448; that is the clamp bound for every fp8 quantisation here (KV cache,
activations), with no per-chip variant."""

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


FP8_CLAMP_MAX: float = 448.0
QUANTIZED_KV_CACHE_DTYPES = ("fp8", "fp8_e4m3")
_KV_DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16, "bf16": torch.bfloat16,
              "fp8": torch.float8_e4m3fn, "fp8_e4m3": torch.float8_e4m3fn}


def kv_cache_dtype_str_to_dtype(kv_cache_dtype: str, model_dtype) -> torch.dtype:
    """``--kv-cache-dtype`` value -> storage dtype of the paged KV cache; ``auto`` keeps the
    model's dtype and the fp8 names map to ``torch.float8_e4m3fn`` (dequantised with the
    per-layer k / v scales inside the attention kernels)."""
    if kv_cache_dtype == "auto":
        return to_torch_dtype(model_dtype)
    if kv_cache_dtype not in _KV_DTYPES:
        raise ValueError(f"unsupported kv_cache_dtype {kv_cache_dtype!r}; supported: 'auto', {sorted(_KV_DTYPES)}")
    return _KV_DTYPES[kv_cache_dtype]
