"""Configuration schema.

``NeuronConfig`` accepts the same ``additional_config["neuron_config"]`` keys as the
Trainium plugin (``vllm_neuron/model/neuron_config.py:117-242``) so a launch
command written for it is accepted unchanged.  On B200 the bucket keys mean CUDA
graph capture sizes (decode) and prefill padding sizes instead of NEFF shapes.

``EngineConfig`` bundles what vLLM spreads over ModelConfig / ParallelConfig /
CacheConfig / SchedulerConfig; the fields keep vLLM's names
(``tensor_parallel_size``, ``max_num_seqs``, ``max_num_batched_tokens``,
``block_size``, ``kv_cache_dtype``, ``enable_prefix_caching`` ...).
"""

from __future__ import annotations

import dataclasses
import json
import os
from dataclasses import dataclass, field
from typing import Any


def _as_bool(v: Any) -> bool:
    if isinstance(v, str):
        return v.lower() in ("true", "1", "yes")
    return bool(v)


class OnDeviceSamplingConfig:
    """On-device sampling knobs (``neuron_config.py:8``)."""

    def __init__(self, **kwargs: Any):
        self.all_greedy = _as_bool(kwargs.pop("all_greedy", False))
        self.max_top_k = int(kwargs.pop("max_top_k", 256))
        self.deterministic = _as_bool(kwargs.pop("deterministic", False))
        self.sampling_dp_degree = int(kwargs.pop("sampling_dp_degree", 1))
        self.capture_topk = _as_bool(kwargs.pop("capture_topk", False))
        if kwargs:
            raise ValueError(f"unknown on_device_sampling_config keys: {sorted(kwargs)}")
        if self.max_top_k < 1:
            raise ValueError("max_top_k must be >= 1")

    def __repr__(self) -> str:
        return f"OnDeviceSamplingConfig({self.__dict__})"


@dataclass
class TensorCaptureConfig:
    modules: list[str] = field(default_factory=list)
    capture_dir: str = "/tmp/vllm_b200_tensor_captures"
    capture_filter: list[str] | None = None


@dataclass
class TensorReplacementConfig:
    tensors: list = field(default_factory=list, repr=False)
    tensors_path: str | None = None
    prompt_token_ids: list | None = field(default=None, repr=False)
    prompt_token_ids_path: str | None = None

    def resolve(self) -> tuple[list, list | None]:
        import torch

        if self.tensors and self.tensors_path:
            raise ValueError("tensor_replacement: specify either 'tensors' or 'tensors_path', not both.")
        tensors = self.tensors or (torch.load(self.tensors_path, weights_only=False) if self.tensors_path else [])
        if not tensors:
            raise ValueError("tensor_replacement: must specify either 'tensors' or 'tensors_path'.")
        ids = self.prompt_token_ids
        if not ids and self.prompt_token_ids_path:
            ids = torch.load(self.prompt_token_ids_path, weights_only=False)
        return tensors, ids


_NEURON_KEYS = (
    "ep_degree", "attention_dp_size", "embedding_dp_size", "lm_head_dp_size", "mlp_dp_size",
    "apply_prefill_dcp", "on_device_sampling_config", "max_logprobs", "prefill_sequence_buckets",
    "decode_batch_buckets", "tensor_capture", "tensor_replacement", "kv_segment_size_buckets",
    "debug_logits_dir", "quantization", "num_batched_tokens_buckets", "num_seqs_buckets",
    "decode_context_length_buckets", "enable_structured_outputs", "fp8_packed_kv",
)


@dataclass
class NeuronConfig:
    """Same keys and defaults as the Trainium plugin's ``NeuronConfig``."""

    ep_degree: int = 1
    attention_dp_size: int = 1
    embedding_dp_size: int = 1
    lm_head_dp_size: int = 1
    mlp_dp_size: int = 1
    # accepted for compatibility: with decode_context_parallel_size > 1 every prefill chunk
    # already attends through the DCP shards (queries gathered, LSE merge), so there is no
    # separate prefill DCP mode to switch on
    apply_prefill_dcp: bool = False
    on_device_sampling_config: OnDeviceSamplingConfig | None = field(default_factory=OnDeviceSamplingConfig)
    max_logprobs: int = 0
    prefill_sequence_buckets: list[int] | None = None
    decode_batch_buckets: list[int] | None = None
    tensor_capture: TensorCaptureConfig | None = None
    tensor_replacement: TensorReplacementConfig | None = None
    kv_segment_size_buckets: list[int] | None = None
    debug_logits_dir: str | None = None
    quantization: str | None = None
    num_batched_tokens_buckets: list[int] | None = None
    num_seqs_buckets: list[int] | None = None
    decode_context_length_buckets: list[int] | None = None
    enable_structured_outputs: bool = False
    fp8_packed_kv: bool = False

    @classmethod
    def from_dict(cls, d: dict | None) -> "NeuronConfig":
        d = dict(d or {})
        unknown = set(d) - set(_NEURON_KEYS)
        if unknown:
            raise ValueError(f"unknown neuron_config keys: {sorted(unknown)}")
        if "on_device_sampling_config" in d:
            ods = d["on_device_sampling_config"]
            d["on_device_sampling_config"] = None if ods is None else (
                ods if isinstance(ods, OnDeviceSamplingConfig) else OnDeviceSamplingConfig(**ods)
            )
        tc = d.get("tensor_capture")
        if isinstance(tc, dict):
            d["tensor_capture"] = TensorCaptureConfig(**tc)
        tr = d.get("tensor_replacement")
        if isinstance(tr, dict):
            d["tensor_replacement"] = TensorReplacementConfig(**tr)
        return cls(**d)

    def __post_init__(self) -> None:
        for k in ("ep_degree", "attention_dp_size", "embedding_dp_size", "lm_head_dp_size", "mlp_dp_size"):
            v = getattr(self, k)
            if not isinstance(v, int) or v < 1:
                raise ValueError(f"{k} must be a positive integer, got {v}")
        if not isinstance(self.enable_structured_outputs, bool):
            raise ValueError(f"enable_structured_outputs must be a boolean, got {self.enable_structured_outputs}")
        if self.quantization not in (None, "bf16", "mxfp4", "fp8", "block_fp8"):
            raise ValueError(f"unsupported quantization {self.quantization!r}")


@dataclass
class VisionNeuronConfig:
    """Vision-encoder knobs (``neuron_config.py:274-450``)."""

    num_vision_tokens_buckets: list[int] | None = None
    vision_attention_block_size: int = 2048
    tp_size: int | None = None
    dp_size: int | None = None
    max_vision_seq_len: int | None = None
    encoder_cache_num_blocks: int | None = None
    encoder_cache_min_hold_time_ms: float = 0.0

    @classmethod
    def from_dict(cls, d: dict | None) -> "VisionNeuronConfig":
        return cls(**(d or {}))

    def resolve_tp_dp(self, world_size: int) -> tuple[int, int]:
        """Vision TP x DP must tile the world (``neuron_config.py:340``)."""
        tp, dp = self.tp_size, self.dp_size
        if tp is None and dp is None:
            tp, dp = world_size, 1
        elif tp is None:
            tp = world_size // dp
        elif dp is None:
            dp = world_size // tp
        if tp * dp != world_size:
            raise ValueError(f"vision tp({tp}) x dp({dp}) must equal world size {world_size}")
        return tp, dp


@dataclass
class SpeculativeConfig:
    method: str = "eagle3"
    model: str | None = None
    num_speculative_tokens: int = 3
    draft_hf_config: Any = None


@dataclass
class KVTransferConfig:
    """Disaggregated prefill/decode (``kv_transfer_config`` of vLLM)."""

    kv_connector: str = "B200IpcConnector"
    kv_role: str = "kv_both"  # kv_producer | kv_consumer | kv_both
    kv_rank: int | None = None
    kv_parallel_size: int = 2
    kv_buffer_device: str = "cuda"
    kv_connector_extra_config: dict = field(default_factory=dict)

    @property
    def is_producer(self) -> bool:
        return self.kv_role in ("kv_producer", "kv_both")

    @property
    def is_consumer(self) -> bool:
        return self.kv_role in ("kv_consumer", "kv_both")


@dataclass
class EngineConfig:
    model: str | None = None
    hf_config: Any = None
    dtype: str = "bfloat16"
    seed: int = 0
    load_format: str = "auto"  # auto | safetensors | dummy
    tensor_parallel_size: int = 1
    data_parallel_size: int = 1
    decode_context_parallel_size: int = 1
    enable_expert_parallel: bool = False
    # EP token exchange of MoE layers under data parallelism: "allgather_reducescatter"
    # (gather every replica's tokens, reduce-scatter the outputs) or an all-to-all that
    # sends each token only to the ranks owning its experts: "neuron" / "b200" (fused NVLink
    # kernels on GPU), "naive" (collective all-to-all)
    all2all_backend: str = "allgather_reducescatter"
    max_model_len: int = 8192
    max_num_seqs: int = 64
    max_num_batched_tokens: int = 4096
    block_size: int = 32
    kv_cache_dtype: str = "auto"  # auto | fp8 | fp8_e4m3
    gpu_memory_utilization: float = 0.90
    num_gpu_blocks_override: int | None = None
    enable_prefix_caching: bool = False
    enable_chunked_prefill: bool = True
    max_num_prefills_per_step: int = 1
    # > 0: prompt chunks of at most this many tokens join the decode steps while requests are
    # decoding (mixed steps); 0: prefill and decode always run as separate steps
    mixed_prefill_tokens: int = 0
    enforce_eager: bool = False
    async_scheduling: bool = False
    device: str = "auto"
    speculative_config: SpeculativeConfig | None = None
    kv_transfer_config: KVTransferConfig | None = None
    neuron_config: NeuronConfig = field(default_factory=NeuronConfig)
    vision_neuron_config: VisionNeuronConfig = field(default_factory=VisionNeuronConfig)
    mm_language_model_only: bool = False
    served_model_name: str | None = None
    profiler_config: dict | None = None

    @classmethod
    def create(cls, **kwargs: Any) -> "EngineConfig":
        extra = kwargs.pop("additional_config", None) or {}
        if isinstance(extra, str):
            extra = json.loads(extra)
        known = {f.name for f in dataclasses.fields(cls)}
        unknown = set(kwargs) - known
        if unknown:
            raise TypeError(f"unknown engine arguments: {sorted(unknown)}")
        cfg = cls(**kwargs)
        if "neuron_config" in extra:
            cfg.neuron_config = NeuronConfig.from_dict(extra["neuron_config"])
        if "vision_neuron_config" in extra:
            cfg.vision_neuron_config = VisionNeuronConfig.from_dict(extra["vision_neuron_config"])
        prof = extra.get("neuron_profiler", extra.get("profiler"))
        if prof is not None:
            from .profiler import ProfilerConfig

            ProfilerConfig.from_dict(prof)  # validate early
            cfg.profiler_config = dict(prof)
        if "mm_language_model_only" in extra:
            cfg.mm_language_model_only = bool(extra["mm_language_model_only"])
        if isinstance(cfg.speculative_config, dict):
            cfg.speculative_config = SpeculativeConfig(**cfg.speculative_config)
        if isinstance(cfg.kv_transfer_config, dict):
            cfg.kv_transfer_config = KVTransferConfig(**cfg.kv_transfer_config)
        cfg.validate()
        return cfg

    @property
    def world_size(self) -> int:
        return self.tensor_parallel_size * self.data_parallel_size

    @property
    def kv_dtype_is_fp8(self) -> bool:
        return self.kv_cache_dtype.startswith("fp8")

    def resolve_device(self) -> str:
        import torch

        from . import envs

        if self.device != "auto":
            return self.device
        if envs.VLLM_B200_CPU_MODE or not torch.cuda.is_available():
            return "cpu"
        return "cuda"

    def expert_parallel_degree(self) -> int:
        """Expert partitions (``neuron_worker.py:88`` resolve_ep_degree): an explicit
        ``neuron_config.ep_degree`` > 1 (variable EP: the ranks of a partition split the
        intermediate dimension), else every rank with ``enable_expert_parallel`` (the
        default EP = TP x DP), else 1 (MoE tensor parallelism over every rank)."""
        nc = self.neuron_config
        if nc.ep_degree > 1:
            return nc.ep_degree
        return self.world_size if self.enable_expert_parallel else 1

    def validate(self) -> None:
        """Checks mirrored from ``NeuronPlatform.check_and_update_config`` (``platform.py:278-393``)."""
        if self.block_size <= 0 or self.block_size & (self.block_size - 1):
            raise ValueError(f"block_size must be a power of two, got {self.block_size}")
        if self.max_num_batched_tokens < 1 or self.max_num_seqs < 1:
            raise ValueError("max_num_batched_tokens and max_num_seqs must be >= 1")
        if not self.enable_chunked_prefill and self.max_num_batched_tokens < self.max_model_len:
            raise ValueError("max_num_batched_tokens < max_model_len requires chunked (segmented) prefill")
        nc = self.neuron_config
        if nc.ep_degree > 1 and self.world_size % nc.ep_degree:
            raise ValueError(f"world size {self.world_size} must be divisible by ep_degree {nc.ep_degree}")
        from .parallel.all2all import A2A_BACKENDS

        if self.all2all_backend not in A2A_BACKENDS:
            raise ValueError(f"all2all_backend must be one of {A2A_BACKENDS}, got {self.all2all_backend!r}")
        if (self.all2all_backend != "allgather_reducescatter" and self.world_size > 1
                and self.expert_parallel_degree() != self.world_size):
            raise ValueError("the EP all-to-all needs every rank to own whole experts: enable expert "
                             "parallelism over all ranks (enable_expert_parallel, or ep_degree = world size)")
        if self.decode_context_parallel_size > 1 and self.tensor_parallel_size % self.decode_context_parallel_size:
            raise ValueError("decode_context_parallel_size must divide tensor_parallel_size")
        if self.kv_cache_dtype not in ("auto", "bf16", "bfloat16", "fp8", "fp8_e4m3"):
            raise ValueError(f"unsupported kv_cache_dtype {self.kv_cache_dtype!r}")
        if self.speculative_config is not None and self.async_scheduling:
            raise ValueError("EAGLE3 speculative decoding and async scheduling are mutually exclusive")

    def to_dict(self) -> dict:
        out = {}
        for f in dataclasses.fields(self):
            v = getattr(self, f.name)
            if f.name == "hf_config":
                continue
            out[f.name] = v if isinstance(v, (int, float, str, bool, type(None))) else repr(v)
        return out


def load_hf_config(model: str) -> dict:
    path = os.path.join(model, "config.json")
    with open(path) as f:
        return json.load(f)
