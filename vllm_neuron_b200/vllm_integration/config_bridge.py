"""vLLM ``VllmConfig`` -> this framework's ``EngineConfig``.

The fields map one to one where both sides have them (model path, dtype, lengths, batch
limits, block size, KV dtype, memory fraction, TP / EP, seed, eager mode); the
``additional_config`` block (``neuron_config``, ``vision_neuron_config``) is passed through
unchanged and validated by the same schema as ``vllm-b200 serve`` uses.  vLLM runs
data-parallel replicas as separate engine cores, so each worker group here is one replica
(``data_parallel_size`` 1).
"""

from __future__ import annotations

from typing import Any

from ..config import EngineConfig


def _dtype_name(dtype: Any) -> str:
    s = str(dtype).replace("torch.", "")
    return {"bfloat16": "bfloat16", "float16": "float16", "half": "float16", "float32": "float32",
            "float": "float32"}.get(s, "bfloat16")


def engine_config_from_vllm(vllm_config: Any, device: str = "auto") -> EngineConfig:
    mc = vllm_config.model_config
    cc = vllm_config.cache_config
    sc = vllm_config.scheduler_config
    pc = vllm_config.parallel_config
    lc = getattr(vllm_config, "load_config", None)
    load_format = str(getattr(lc, "load_format", "auto") or "auto")
    if load_format not in ("auto", "safetensors", "dummy"):
        load_format = "auto"
    extra = getattr(vllm_config, "additional_config", None) or {}
    served = getattr(mc, "served_model_name", None)
    if isinstance(served, (list, tuple)):
        served = served[0] if served else None
    kv_dtype = str(getattr(cc, "cache_dtype", "auto") or "auto")
    kw = dict(
        model=mc.model,
        dtype=_dtype_name(mc.dtype),
        seed=int(getattr(mc, "seed", 0) or 0),
        load_format=load_format,
        tensor_parallel_size=int(pc.tensor_parallel_size),
        data_parallel_size=1,
        enable_expert_parallel=bool(getattr(pc, "enable_expert_parallel", False)),
        max_model_len=int(mc.max_model_len),
        max_num_seqs=int(sc.max_num_seqs),
        max_num_batched_tokens=int(sc.max_num_batched_tokens),
        block_size=int(cc.block_size or 32),
        kv_cache_dtype=kv_dtype if kv_dtype.startswith("fp8") else "auto",
        gpu_memory_utilization=float(cc.gpu_memory_utilization),
        num_gpu_blocks_override=getattr(cc, "num_gpu_blocks_override", None),
        enable_prefix_caching=bool(getattr(cc, "enable_prefix_caching", False)),
        enforce_eager=bool(getattr(mc, "enforce_eager", False)),
        async_scheduling=False,  # the worker returns each step's tokens before the next step
        device=device,
        served_model_name=served,
        additional_config=dict(extra) if isinstance(extra, dict) else extra,
    )
    return EngineConfig.create(**kw)
