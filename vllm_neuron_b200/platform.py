"""vLLM platform-plugin hook.

``vllm_neuron_b200.register()`` is the ``vllm.platform_plugins`` entry point (the
Trainium plugin's ``vllm_neuron:register``, ``vllm_neuron/__init__.py:201``).  It returns
the path of :class:`B200Platform`, a subclass of vLLM's CUDA platform that validates the
``additional_config["neuron_config"]`` block with this framework's schema, applies its
defaults (block size 32, the reference's default) and installs this framework's worker and
scheduler into vLLM's configuration (``vllm/platform.py:322-325`` and ``:376-387`` of the
reference): ``parallel_config.worker_cls`` becomes
:class:`vllm_neuron_b200.vllm_integration.worker.B200VllmWorker` and
``scheduler_config.scheduler_cls`` the matching class of
``vllm_neuron_b200.vllm_integration.scheduler``, so ``vllm serve`` with this plugin runs the
model, kernels and collectives of this framework under vLLM's front end, request queue and
KV block manager.  A worker or scheduler class the user configured explicitly is kept.
"""

from __future__ import annotations

PLATFORM_PATH = "vllm_neuron_b200.platform.B200Platform"
WORKER_CLS = "vllm_neuron_b200.vllm_integration.worker.B200VllmWorker"
SCHEDULER_CLS = "vllm_neuron_b200.vllm_integration.scheduler.B200VllmScheduler"
ASYNC_SCHEDULER_CLS = "vllm_neuron_b200.vllm_integration.scheduler.B200VllmAsyncScheduler"
_VLLM_SCHEDULERS = (None, "vllm.v1.core.sched.scheduler.Scheduler",
                    "vllm.v1.core.sched.async_scheduler.AsyncScheduler")


def install_worker_and_scheduler(vllm_config) -> None:
    """Point vLLM at this framework's worker and scheduler (explicit user choices kept)."""
    pc = getattr(vllm_config, "parallel_config", None)
    if pc is not None and getattr(pc, "worker_cls", "auto") == "auto":
        pc.worker_cls = WORKER_CLS
    sc = getattr(vllm_config, "scheduler_config", None)
    if sc is not None and getattr(sc, "scheduler_cls", None) in _VLLM_SCHEDULERS + (SCHEDULER_CLS,
                                                                                   ASYNC_SCHEDULER_CLS):
        sc.scheduler_cls = ASYNC_SCHEDULER_CLS if getattr(sc, "async_scheduling", False) else SCHEDULER_CLS


def get_platform_class() -> str:
    return PLATFORM_PATH


def _platform_base():
    """vLLM's CUDA platform; on a host without the CUDA driver (vLLM's CUDA platform cannot
    load there) vLLM's CPU platform, under which this framework's worker runs its CPU path."""
    try:
        from vllm.platforms.cuda import CudaPlatform

        return CudaPlatform
    except Exception:  # noqa: BLE001 - no CUDA driver, or vLLM absent
        pass
    try:
        from vllm.platforms.cpu import CpuPlatform

        return CpuPlatform
    except Exception:  # noqa: BLE001 - vLLM absent or not importable: plain marker class
        class _Marker:
            device_name = "cuda"

            @classmethod
            def check_and_update_config(cls, vllm_config) -> None:  # pragma: no cover
                return None

        return _Marker


def _make_platform(base=None):
    CudaPlatform = base if base is not None else _platform_base()  # noqa: N806

    class B200Platform(CudaPlatform):  # type: ignore[misc,valid-type]
        device_name = getattr(CudaPlatform, "device_name", "cuda")
        default_block_size = 32

        @classmethod
        def get_attn_backend_cls(cls, *args, **kwargs) -> str:  # ``platform.py:663`` of the reference
            return "vllm_neuron_b200.ops.metadata.B200AttentionBackend"

        @classmethod
        def check_and_update_config(cls, vllm_config) -> None:
            from .config import NeuronConfig

            extra = getattr(vllm_config, "additional_config", None) or {}
            if isinstance(extra, dict) and "neuron_config" in extra:
                NeuronConfig.from_dict(extra["neuron_config"])  # raises on invalid keys / values
            cache = getattr(vllm_config, "cache_config", None)
            if cache is not None and getattr(cache, "block_size", None) in (None, 0):
                cache.block_size = cls.default_block_size
            install_worker_and_scheduler(vllm_config)
            parent = getattr(super(), "check_and_update_config", None)
            if parent is not None:
                parent(vllm_config)

    return B200Platform


def __getattr__(name):
    if name == "B200Platform":
        cls = _make_platform()
        globals()["B200Platform"] = cls
        return cls
    raise AttributeError(name)
