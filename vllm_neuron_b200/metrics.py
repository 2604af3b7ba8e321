"""Prometheus metrics (parity with ``vllm_neuron/metrics.py:23-69``).

Same shapes and labels as the Trainium plugin's metrics, under the ``vllm_b200:``
prefix.  ``graph_replay_count`` replaces the NEFF execution counter: one decode
step replays one captured CUDA graph per (batch bucket).  When
``prometheus_client`` is unavailable every metric is a no-op object so the
engine never depends on it.
"""

from __future__ import annotations

from typing import Any

try:  # pragma: no cover - import guard
    from prometheus_client import Counter, Gauge, Histogram

    _HAVE_PROM = True
except Exception:  # pragma: no cover
    _HAVE_PROM = False


class _Noop:
    def labels(self, *a: Any, **k: Any) -> "_Noop":
        return self

    def observe(self, *a: Any, **k: Any) -> None:
        pass

    def inc(self, *a: Any, **k: Any) -> None:
        pass

    def set(self, *a: Any, **k: Any) -> None:
        pass


_PADDING_BUCKETS = (0, 1, 2, 4, 8, 16, 32, 64, 128, 256, 512, 1024, 2048, 4096)


def _make(kind: str, name: str, doc: str, labels: tuple[str, ...], **kw: Any):
    if not _HAVE_PROM:
        return _Noop()
    cls = {"h": Histogram, "c": Counter, "g": Gauge}[kind]
    try:
        return cls(name, doc, labels, **kw)
    except ValueError:  # already registered (module reloaded in tests)
        from prometheus_client import REGISTRY

        return REGISTRY._names_to_collectors.get(name, _Noop())  # type: ignore[attr-defined]


NUM_SEQS_PADDING = _make(
    "h", "vllm_b200:num_seqs_padding", "Padding sequences added to reach a decode batch bucket", ("model_name",),
    buckets=_PADDING_BUCKETS,
)
NUM_BATCHED_TOKENS_PADDING = _make(
    "h", "vllm_b200:num_batched_tokens_padding", "Padding tokens added to reach a prefill bucket", ("model_name",),
    buckets=_PADDING_BUCKETS,
)
GRAPH_REPLAY_COUNT = _make(
    "c", "vllm_b200:graph_replay_count", "CUDA-graph replays per bucket", ("model_name", "bucket_name")
)
COMPILATION_TIME = _make("g", "vllm_b200:compilation_time_seconds", "Graph capture time", ("model_name",))
STARTUP_TIME = _make("g", "vllm_b200:startup_time_seconds", "Worker start-up time", ("model_name",))
MODEL_LOAD_TIME = _make("g", "vllm_b200:model_load_time_seconds", "Weight load time", ("model_name",))
MODEL_LOAD_SIZE = _make("g", "vllm_b200:model_load_size_bytes", "Bytes of weights loaded", ("model_name",))
ASYNC_STEPS = _make(
    "c", "vllm_b200:async_steps", "Engine steps under asynchronous scheduling by how they ran: launched (pipeline "
    "started), lookahead (scheduled while the previous step ran), sync_fallback (drained and run synchronously)",
    ("model_name", "mode"))
NVLINK_BYTES = _make("c", "vllm_b200:nvlink_bytes", "Bytes moved by fused collectives", ("model_name", "op"))
