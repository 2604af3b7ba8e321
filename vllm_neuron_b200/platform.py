"""vLLM platform-plugin hook.

``vllm_neuron_b200.register()`` is the ``vllm.platform_plugins`` entry point (the
Trainium plugin's ``vllm_neuron:register``, ``vllm_neuron/__init__.py:201``).  It returns
the path of :class:`B200Platform`, a subclass of vLLM's CUDA platform that validates the
``additional_config["neuron_config"]`` block with this framework's schema and applies
its defaults (block size 32, the reference's default).  Serving itself runs on this
framework's engine (``vllm-b200 serve`` / :class:`vllm_neuron_b200.LLM`), whose kernels and
scheduler replace vLLM's.
"""

from __future__ import annotations

PLATFORM_PATH = "vllm_neuron_b200.platform.B200Platform"


def get_platform_class() -> str:
    return PLATFORM_PATH


def _make_platform():
    try:
        from vllm.platforms.cuda import CudaPlatform
    except Exception:  # noqa: BLE001 - vLLM absent or not importable: plain marker class
        class CudaPlatform:  # type: ignore[no-redef]
            device_name = "cuda"

            @classmethod
            def check_and_update_config(cls, vllm_config) -> None:  # pragma: no cover
                return None

    class B200Platform(CudaPlatform):  # type: ignore[misc,valid-type]
        device_name = "cuda"
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
