"""Environment-variable registry for the B200 framework.

Every variable is read lazily (at attribute access), so tests can flip them with
``monkeypatch.setenv`` without re-importing.  Names use the ``VLLM_B200_`` prefix;
where the Trainium plugin had an equivalent knob (``vllm_neuron/envs.py:117-255``)
the ``VLLM_NEURON_`` spelling is accepted as an alias so existing launch scripts
keep working.

Knobs that only made sense for the Neuron compiler (NEFF cache, parallel trace,
HLO dumps) have no counterpart: kernels are compiled ahead of time by nvcc and
decode steps are replayed as CUDA graphs.
"""

from __future__ import annotations

import os
from typing import Any, Callable


def _bool(v: str) -> bool:
    return v.strip().lower() in ("1", "true", "yes", "on")


def _get(name: str, default: str | None, alias: str | None = None) -> str | None:
    if name in os.environ:
        return os.environ[name]
    if alias is not None and alias in os.environ:
        return os.environ[alias]
    return default


# name -> (parser, default, alias)
_REGISTRY: dict[str, tuple[Callable[[str], Any], str | None, str | None]] = {
    # Run every op through its PyTorch reference implementation (CPU mode).
    "VLLM_B200_CPU_MODE": (_bool, "0", "VLLM_NEURON_CPU_MODE"),
    # Disable the hand-written CUDA kernels (use the PyTorch reference ops on GPU).
    "VLLM_B200_DISABLE_KERNELS": (_bool, "0", "VLLM_NEURON_DISABLE_NKI_KERNELS"),
    # Disable CUDA-graph capture of decode buckets (eager decode).
    "VLLM_B200_DISABLE_CUDA_GRAPHS": (_bool, "0", "VLLM_NEURON_DISABLE_GRAPH_CAPTURE_BACKEND"),
    # Logging level of the ``vllm_neuron_b200`` logger.
    "VLLM_B200_LOG_LEVEL": (str, "INFO", "VLLM_NEURON_LOG_LEVEL"),
    # Debug mode: host-side validation of block tables / slot mappings before launch,
    # device status words checked after every step.
    "VLLM_B200_DEBUG_MODE": (_bool, "0", "VLLM_NEURON_DEBUG_MODE"),
    # Barrier / process-group timeout in seconds.
    "VLLM_B200_BARRIER_TIMEOUT": (int, "3600", "VLLM_NEURON_BARRIER_TIMEOUT"),
    # Minimum KV-cache budget in GiB; below it the worker fails fast.
    "VLLM_B200_MIN_KV_BUDGET_GIB": (float, "1.0", "VLLM_NEURON_MIN_KV_BUDGET_GIB"),
    # Skip warm-up (graph capture) of the decode buckets.  Prefill runs eagerly (no per-bucket
    # graphs), so the prefill switch is accepted for compatibility and has nothing to skip.
    "VLLM_B200_SKIP_PREFILL_WARMUP": (_bool, "0", "VLLM_NEURON_SKIP_PREFILL_WARMUP"),
    "VLLM_B200_SKIP_DECODE_WARMUP": (_bool, "0", "VLLM_NEURON_SKIP_DECODE_WARMUP"),
    # Seconds a worker gets between SIGTERM and SIGKILL at shutdown.
    "VLLM_B200_WORKER_TERMINATION_TIMEOUT": (float, "5", "VLLM_NEURON_WORKER_TERMINATION_TIMEOUT"),
    # Gate the synthetic KV-verification model into the registry (DI tests).
    "VLLM_B200_SYNTHETIC_MODEL": (_bool, "0", "VLLM_NEURON_SYNTHETIC_MODEL"),
    # sequence parallelism for TP prefill steps (token rows split across TP between blocks)
    "VLLM_B200_SEQUENCE_PARALLEL": (_bool, "1", None),
    # Directory for golden logits used by accuracy tests.
    "VLLM_B200_GOLDEN_CACHE_DIR": (str, "", "VLLM_NEURON_GOLDEN_CACHE_DIR"),
    # Use the fused in-kernel NVLink collectives (else NCCL).
    "VLLM_B200_FUSED_COLLECTIVES": (_bool, "1", None),
    # Row-parallel GEMMs reduce their output tiles through NVSwitch (multimem) when the group
    # has a multicast object (else the GEMM and the fused all-reduce kernel run separately).
    "VLLM_B200_GEMM_ALLREDUCE": (_bool, "0", None),
    # The decode all-reduce kernel sends LL units (data with the call's epoch in every 16-byte
    # store) instead of data + one release flag per peer.
    "VLLM_B200_AR_LL": (_bool, "1", None),
    # The MoE layer's per-token route sum runs inside the layer-boundary collective kernel.
    "VLLM_B200_FUSE_MOE_ROUTE_SUM": (_bool, "1", None),
    # Sequence-parallel prefill boundaries as one NVLink kernel (reduce-scatter + norm +
    # all-gather), fed by the row-parallel GEMM's scattered stores (else NCCL + the norm).
    "VLLM_B200_FUSED_SP": (_bool, "1", None),
    # Sliding-window layers keep their own KV block pool (blocks behind the window are freed).
    "VLLM_B200_SWA_KV_GROUP": (_bool, "1", None),
    # Dense layers through the library GEMM (torch / cuBLAS) instead of the tcgen05 kernel:
    # the NCCL + cuBLAS baseline-of-record configuration, never the default.
    "VLLM_B200_LIBRARY_GEMM": (_bool, "0", None),
    # Spin-wait bound (iterations) for device-side flag waits in fused collectives.
    "VLLM_B200_DEVICE_WAIT_LIMIT": (int, "20000000", None),
    # Prometheus multiprocess directory (set automatically when unset).
    "PROMETHEUS_MULTIPROC_DIR": (str, "", None),
    # First GPU index of this engine (rank r uses GPU offset + r).
    "VLLM_B200_DEVICE_OFFSET": (int, "0", None),
    # Pin each rank's threads to the CPUs of its GPU's NUMA node.
    "VLLM_B200_CPU_AFFINITY": (_bool, "0", None),
    # Bidirectional KV transfer for disaggregated serving.
    "VLLM_B200_BIDIRECTIONAL_KV": (_bool, "0", "VLLM_NEURON_BIDIRECTIONAL_KV"),
}


def __getattr__(name: str) -> Any:
    if name in _REGISTRY:
        parser, default, alias = _REGISTRY[name]
        raw = _get(name, default, alias)
        return parser(raw) if raw is not None else None
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")


def __dir__() -> list[str]:
    return sorted(_REGISTRY)


def snapshot() -> dict[str, Any]:
    """Current value of every registered variable (for logging at start-up)."""
    return {k: __getattr__(k) for k in _REGISTRY}


def get_dist_backend() -> str:
    """Device collective backend: NCCL on GPU, gloo in CPU mode."""
    import torch

    if __getattr__("VLLM_B200_CPU_MODE") or not torch.cuda.is_available():
        return "gloo"
    return "nccl"
