"""Loader for the compiled sm_100a extension (``vllm_neuron_b200/_C*.so``).

The extension registers its kernels as ``torch.ops.b200.*``.  It is built in-tree by
``python setup.py build_ext --inplace``.  On a CUDA tensor the ops layer requires
it: a missing extension raises instead of silently running the PyTorch reference,
unless ``VLLM_B200_DISABLE_KERNELS=1`` asks for the reference path explicitly.
"""

from __future__ import annotations

import importlib
import os

import torch

_LOADED: bool | None = None
_ERR: str | None = None


def load() -> bool:
    global _LOADED, _ERR
    if _LOADED is not None:
        return _LOADED
    try:
        importlib.import_module("vllm_neuron_b200._C")
        _LOADED = hasattr(torch.ops, "b200") and hasattr(torch.ops.b200, "rms_norm")
        if not _LOADED:
            _ERR = "extension imported but torch.ops.b200 is not registered"
    except Exception as e:  # noqa: BLE001
        _LOADED, _ERR = False, f"{type(e).__name__}: {e}"
    return _LOADED


def load_error() -> str | None:
    load()
    return _ERR


def so_path() -> str | None:
    try:
        mod = importlib.import_module("vllm_neuron_b200._C")
        return os.path.abspath(mod.__file__)
    except Exception:  # noqa: BLE001
        return None


def kernels_enabled() -> bool:
    from .. import envs

    return not envs.VLLM_B200_DISABLE_KERNELS and not envs.VLLM_B200_CPU_MODE


def use_kernel(t: torch.Tensor) -> bool:
    """True when ``t`` lives on a GPU and kernels are enabled.  Raises when the
    extension that should run is missing."""
    if not t.is_cuda or not kernels_enabled():
        return False
    if not load():
        raise RuntimeError(
            "vllm_neuron_b200 CUDA extension is not available on a GPU tensor "
            f"({_ERR}); build it with `python setup.py build_ext --inplace` or set "
            "VLLM_B200_DISABLE_KERNELS=1 to run the PyTorch reference ops"
        )
    return True


class _DebugOps:
    """``VLLM_B200_DEBUG_SYNC=1``: every kernel call synchronises and checks both the
    CUDA error state and the kernel status word, naming the op that failed."""

    def __getattr__(self, name):
        fn = getattr(torch.ops.b200, name)

        def call(*args, **kwargs):
            out = fn(*args, **kwargs)
            try:
                torch.cuda.synchronize()
            except Exception as e:  # noqa: BLE001
                raise RuntimeError(f"b200::{name} failed: {e}") from e
            from . import check_device_status

            for a in args:
                if isinstance(a, torch.Tensor) and a.is_cuda:
                    try:
                        check_device_status(a.device)
                    except RuntimeError as e:
                        raise RuntimeError(f"b200::{name}: {e}") from e
                    break
            return out

        return call


_DEBUG = _DebugOps()


def ops():
    load()
    if os.environ.get("VLLM_B200_DEBUG_SYNC", "0") == "1":
        return _DEBUG
    return torch.ops.b200
