"""vllm_neuron_b200: a Blackwell (sm_100a) serving framework with the feature set of
the vllm-neuron plugin.

Public API:
    LLM, SamplingParams, RequestOutput   offline inference (``vllm.LLM``-compatible)
    EngineConfig, NeuronConfig            configuration (same ``neuron_config`` keys)
    register()                            vLLM platform-plugin entry point
"""

from __future__ import annotations

__version__ = "0.1.0"

from .config import EngineConfig, NeuronConfig  # noqa: E402,F401
from .engine.sampling_params import RequestOutput, SamplingParams  # noqa: E402,F401


def __getattr__(name):
    if name == "LLM":
        from .engine.llm import LLM

        return LLM
    if name == "LLMEngine":
        from .engine.llm_engine import LLMEngine

        return LLMEngine
    raise AttributeError(name)


def register() -> str:
    """vLLM ``vllm.platform_plugins`` entry point: returns the platform class path
    (``vllm_neuron/__init__.py:201``)."""
    from .platform import get_platform_class

    return get_platform_class()
