"""Model registry: HF architecture name -> (model class, config class)
(``vllm_neuron/model/registry.py:10``)."""

from __future__ import annotations

import importlib

from .. import envs

_MODELS: dict[str, tuple[str, str, str]] = {
    # arch: (module, model class, config class)
    "GptOssForCausalLM": ("gpt_oss", "GptOssForCausalLM", "GptOssConfig"),
    "LlamaForCausalLM": ("llama", "LlamaForCausalLM", "LlamaConfig"),
    "Eagle3LlamaForCausalLM": ("eagle3", "Eagle3LlamaForCausalLM", "Eagle3Config"),
    "Qwen3VLForConditionalGeneration": ("qwen3_vl", "Qwen3VLForConditionalGeneration", "Qwen3VLConfig"),
    "Qwen3NextForCausalLM": ("qwen3_next", "Qwen3NextForCausalLM", "Qwen3NextConfig"),
}
_SYNTHETIC = {"SyntheticModel": ("synthetic", "SyntheticModel", "SyntheticConfig"),
              "SyntheticNeuronModel": ("synthetic", "SyntheticModel", "SyntheticConfig")}


def get_models() -> dict[str, tuple[str, str, str]]:
    m = dict(_MODELS)
    if envs.VLLM_B200_SYNTHETIC_MODEL:
        m.update(_SYNTHETIC)
    return m


def resolve(hf: dict) -> tuple[type, type]:
    archs = hf.get("architectures") or []
    models = get_models()
    for a in archs:
        if a in models:
            mod, cls, cfg = models[a]
            m = importlib.import_module(f"vllm_neuron_b200.models.{mod}")
            return getattr(m, cls), getattr(m, cfg)
    raise ValueError(f"unsupported architectures {archs}; supported: {sorted(models)}")
