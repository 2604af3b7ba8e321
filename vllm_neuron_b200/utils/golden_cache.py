"""On-disk cache of reference ("golden") outputs (``utils/golden_cache.py`` of the Trainium plugin).

Reference model runs (e.g. HF fp32 generations or logits) are slow; tests and accuracy tools
key them by a hash of everything that determines them (model config, prompts, generation
parameters, library versions) and reuse them.  ``VLLM_B200_GOLDEN_CACHE_DIR`` (alias
``VLLM_NEURON_GOLDEN_CACHE_DIR``) sets the directory (default ``~/.cache/vllm_b200/golden``);
the value ``off`` disables the cache.
"""

from __future__ import annotations

import hashlib
import json
import os
from typing import Any, Callable

import torch


def cache_dir() -> str | None:
    d = (os.environ.get("VLLM_B200_GOLDEN_CACHE_DIR") or os.environ.get("VLLM_NEURON_GOLDEN_CACHE_DIR")
         or os.path.join(os.path.expanduser("~"), ".cache", "vllm_b200", "golden"))
    return None if d.lower() in ("off", "0", "none", "") else d


def golden_key(**parts: Any) -> str:
    import transformers

    blob = json.dumps({"v": [torch.__version__, transformers.__version__], **parts}, sort_keys=True, default=str)
    return hashlib.sha256(blob.encode()).hexdigest()[:24]


def get_or_compute(key: str, fn: Callable[[], Any]) -> Any:
    d = cache_dir()
    if d is None:
        return fn()
    path = os.path.join(d, f"{key}.pt")
    if os.path.exists(path):
        try:
            return torch.load(path, weights_only=False)
        except Exception:  # noqa: BLE001  (truncated file: recompute)
            pass
    val = fn()
    os.makedirs(d, exist_ok=True)
    tmp = f"{path}.tmp{os.getpid()}"
    torch.save(val, tmp)
    os.replace(tmp, path)
    return val
