"""One worker per GPU: device and process-group set-up, model load, KV budget,
warm-up (decode graph capture) and step execution.

Counterpart of ``NeuronWorker`` (``vllm_neuron/vllm/worker/neuron_worker.py:188``):
* the KV budget is what is left after weights and an activation reserve at the
  configured ``gpu_memory_utilization``, min-reduced over ranks so every rank
  allocates the same number of blocks, and must reach ``VLLM_B200_MIN_KV_BUDGET_GIB``
  (fail fast, ``neuron_worker.py:777-787``);
* warm-up captures one CUDA graph per decode bucket (``VLLM_B200_SKIP_DECODE_WARMUP``
  skips it; graphs are then captured lazily on first use).
"""

from __future__ import annotations

import math
import os
import time

import torch

from .. import envs
from ..config import EngineConfig, load_hf_config
from ..logging_config import init_logger
from ..metrics import MODEL_LOAD_SIZE, MODEL_LOAD_TIME, STARTUP_TIME
from ..models.base import random_init_, random_init_device_
from ..models.registry import resolve
from ..parallel import state as pstate
from ..utils.dtype_utils import kv_cache_dtype_str_to_dtype
from .model_runner import ModelRunner

logger = init_logger(__name__)


def build_model(cfg: EngineConfig, ps, device: torch.device, hf: dict | None = None):
    hf = hf if hf is not None else (cfg.hf_config if isinstance(cfg.hf_config, dict) else load_hf_config(cfg.model))
    model_cls, config_cls = resolve(hf)
    mcfg = config_cls.from_hf(hf, quantization=cfg.neuron_config.quantization)
    dtype = torch.bfloat16 if cfg.dtype in ("bfloat16", "bf16", "auto") else (
        torch.float32 if cfg.dtype in ("float32", "fp32") else torch.float16)
    # fp8 names select the e4m3fn cache; the 16-bit names keep the model's dtype
    kv_dtype = kv_cache_dtype_str_to_dtype(cfg.kv_cache_dtype, dtype) if cfg.kv_dtype_is_fp8 else dtype
    model = model_cls(mcfg, ps, dtype=dtype, device=device, kv_dtype=kv_dtype)
    return model, mcfg, hf


class Worker:
    def __init__(self, cfg: EngineConfig, rank: int = 0, world_size: int = 1, local_rank: int = 0,
                 init_method: str | None = None):
        self.cfg = cfg
        self.init_method = init_method  # process-group rendezvous (None: file store / env://)
        # the windowed layers may get their own block pool (off when an outer KV manager,
        # such as vLLM's, owns a single block table per request)
        self.swa_group_allowed = True
        self.rank = rank
        self.world_size = world_size
        self.local_rank = local_rank
        # GPU of this rank: local rank + VLLM_B200_DEVICE_OFFSET, so two servers that both see every
        # GPU of the host (CUDA IPC between them needs that) can still sit on disjoint GPUs
        self.device_index = local_rank + envs.VLLM_B200_DEVICE_OFFSET
        self.device = torch.device("cpu")
        self.model = None
        self.runner: ModelRunner | None = None
        self.ps = None

    def init_device(self) -> None:
        t0 = time.time()
        dev = self.cfg.resolve_device()
        if dev == "cuda":
            torch.cuda.set_device(self.device_index)
            self.device = torch.device("cuda", self.device_index)
            if envs.VLLM_B200_CPU_AFFINITY:
                from ..utils.hardware_config import bind_to_gpu_numa

                cpus = bind_to_gpu_numa(self.device_index)
                logger.info("rank %d pinned to %s CPUs of its GPU's NUMA node", self.rank,
                            len(cpus) if cpus else "no (node unknown)")
        pstate.init_distributed_environment(self.world_size, self.rank, init_method=self.init_method,
                                            local_rank=self.device_index,
                                            timeout_s=float(envs.VLLM_B200_BARRIER_TIMEOUT))
        nc = self.cfg.neuron_config
        self.ps = pstate.initialize_parallel_state(
            tp=self.cfg.tensor_parallel_size, dp=self.cfg.data_parallel_size,
            ep_degree=self.cfg.expert_parallel_degree(), attention_dp_size=nc.attention_dp_size,
            embedding_dp_size=nc.embedding_dp_size, lm_head_dp_size=nc.lm_head_dp_size,
            mlp_dp_size=nc.mlp_dp_size, dcp=self.cfg.decode_context_parallel_size,
            vision_tp=self.cfg.vision_neuron_config.tp_size, vision_dp=self.cfg.vision_neuron_config.dp_size,
            timeout_s=float(envs.VLLM_B200_BARRIER_TIMEOUT), sampling_dp=self._sampling_dp())
        if self.device.type == "cuda" and self.world_size > 1 and envs.VLLM_B200_FUSED_COLLECTIVES:
            from ..parallel.communicator import attach_communicators, attach_reducers

            attach_communicators(self.ps, self.device)
            attach_reducers(self.ps, self.device)
        self._t_start = t0

    def load_model(self) -> None:
        t0 = time.time()
        torch.manual_seed(self.cfg.seed)
        model, mcfg, hf = build_model(self.cfg, self.ps, self.device)
        if (self.device.type == "cuda" and self.world_size > 1 and envs.VLLM_B200_FUSED_COLLECTIVES
                and hasattr(mcfg, "hidden_size")):
            from ..parallel.communicator import attach_sp_communicator

            attach_sp_communicator(self.ps, self.device, self.cfg.max_num_batched_tokens, mcfg.hidden_size)
        if self.cfg.load_format == "dummy" or self.cfg.model is None:
            if self.device.type == "cuda":
                random_init_device_(model, self.cfg.seed)
            else:
                random_init_(model, self.cfg.seed)
        else:
            from ..utils.checkpoints import SafetensorsCheckpoint

            ck = SafetensorsCheckpoint(self.cfg.model)
            model.load_weights(((k, v.to(self.device) if v.numel() > (1 << 20) else v) for k, v in ck))
        for m in model.modules():  # kernel weight layouts (e.g. grouped-GEMM tiles)
            if hasattr(m, "process_weights_after_loading"):
                m.process_weights_after_loading()
        if hasattr(model, "vision_block_size"):
            model.vision_block_size = int(self.cfg.vision_neuron_config.vision_attention_block_size)
        self.model = model.eval()
        self.model_cfg = mcfg
        self.hf = hf
        nbytes = sum(p.numel() * p.element_size() for p in model.parameters())
        name = self.cfg.served_model_name or str(self.cfg.model)
        MODEL_LOAD_TIME.labels(model_name=name).set(time.time() - t0)
        MODEL_LOAD_SIZE.labels(model_name=name).set(nbytes)
        vocab = getattr(mcfg, "vocab_size", None) or hf.get("vocab_size")
        nc = self.cfg.neuron_config
        if max(nc.embedding_dp_size, nc.lm_head_dp_size, nc.mlp_dp_size) > 1 and self.cfg.speculative_config:
            raise ValueError("component data parallelism with speculative decoding is not supported")
        if nc.attention_dp_size > 1:
            if not hasattr(model, "attention_dp"):
                raise ValueError(f"attention_dp_size > 1 is not supported for {type(model).__name__}")
            if (nc.attention_dp_size != self.cfg.data_parallel_size or self.cfg.speculative_config
                    or self.cfg.decode_context_parallel_size > 1
                    or max(nc.embedding_dp_size, nc.lm_head_dp_size, nc.mlp_dp_size) > 1):
                raise ValueError("attention_dp_size must equal data_parallel_size, without speculative decoding, "
                                 "DCP or component DP")
        self._attach_all2all(model, mcfg)
        dcp = self.cfg.decode_context_parallel_size
        if dcp > 1:
            self._check_dcp(mcfg, hf, dcp)
        sdp = self._sampling_dp()
        self.runner = ModelRunner(self.cfg, model, self.device, self.ps.tp, vocab,
                                  cp_group=self.ps.dcp_kv if dcp > 1 else None,
                                  sampling_groups=(self.ps.sampling_a2a, self.ps.sampling_gather) if sdp > 1 else None)
        logger.info("rank %d loaded model (%.2f GB) in %.1fs", self.rank, nbytes / 1e9, time.time() - t0)

    def _sampling_dp(self) -> int:
        ods = self.cfg.neuron_config.on_device_sampling_config
        return ods.sampling_dp_degree if ods is not None else 1

    def _attach_all2all(self, model, mcfg) -> None:
        """One EP all-to-all object (over the world group) shared by every MoE layer that
        supports it, when ``all2all_backend`` selects one and experts span several ranks."""
        from ..parallel.all2all import make_ep_all2all

        layers = [m for m in model.modules() if hasattr(m, "a2a")]
        if not layers or self.cfg.all2all_backend == "allgather_reducescatter" or self.ps.world.world_size == 1:
            return
        a2a = make_ep_all2all(self.cfg.all2all_backend, self.ps.world, self.device, mcfg.hidden_size,
                              mcfg.num_experts_per_tok, max_tokens=min(256, self.cfg.max_num_seqs), ps=self.ps)
        for m in layers:
            m.a2a = a2a
        self.a2a = a2a

    def _check_dcp(self, mcfg, hf: dict, dcp: int) -> None:
        """DCP groups are runs of ``dcp`` consecutive TP ranks, which share a KV head under
        the TP sharding exactly when ``(tp // kv_heads) % dcp == 0`` (``platform.py:579-620``
        states the same condition as kv_heads < tp, dcp <= tp / kv_heads)."""
        tp = self.cfg.tensor_parallel_size
        hkv = getattr(mcfg, "num_key_value_heads", None) or hf.get("num_key_value_heads")
        if hasattr(self.model, "get_state_spec"):
            raise ValueError("decode context parallelism does not apply to recurrent (linear-attention) layers")
        if self.cfg.speculative_config is not None:
            raise ValueError("decode context parallelism with speculative decoding is not supported")
        if not hkv or hkv * dcp > tp or (tp // hkv) % dcp:
            raise ValueError(f"decode_context_parallel_size {dcp} needs (tp // kv_heads) % dcp == 0 "
                             f"(tp={tp}, kv_heads={hkv})")

    def swa_group_window(self) -> int | None:
        """The sliding window when the windowed layers get their own KV block pool (models
        mixing sliding-window and full-attention layers; not with prefix caching, DCP, KV
        transfer, speculative decoding, attention DP or recurrent layers, whose block tables
        are shared by every layer)."""
        c = self.cfg
        if not self.swa_group_allowed:
            return None
        if not envs.VLLM_B200_SWA_KV_GROUP or c.enable_prefix_caching or c.decode_context_parallel_size > 1:
            return None
        if c.kv_transfer_config or c.speculative_config is not None or c.neuron_config.attention_dp_size > 1:
            return None
        if self.runner is not None and self.runner.state_caches is not None:
            return None
        return self.model.get_kv_spec().sliding_window

    def swa_blocks_for(self) -> int:
        """Blocks of the sliding-window group: every running sequence holds at most its window
        plus one partial block on each side, and each prefill step's chunk adds its tokens."""
        w = self.swa_group_window()
        if not w:
            return 0
        bs, c = self.cfg.block_size, self.cfg
        per_seq = -(-w // bs) + 2
        chunk = -(-c.max_num_batched_tokens // bs) + 1
        return c.max_num_seqs * per_seq + max(1, c.max_num_prefills_per_step) * chunk + 1

    def determine_num_blocks(self) -> int:
        """Blocks of the full-attention group (``self.num_swa_blocks`` is set for the
        sliding-window group when it is kept apart)."""
        spec = self.model.get_kv_spec()
        self.num_swa_blocks = self.swa_blocks_for()
        per_block = max(1, spec.bytes_per_block(self.cfg.block_size, False if self.num_swa_blocks else None))
        swa_bytes = self.num_swa_blocks * spec.bytes_per_block(self.cfg.block_size, True) if self.num_swa_blocks else 0
        # a (virtual) block of a DCP rank holds block_size of its group's bs * dcp tokens
        vbs = self.cfg.block_size * self.cfg.decode_context_parallel_size
        need = self.cfg.max_num_seqs * math.ceil(self.cfg.max_model_len / vbs) + 1
        if self.cfg.num_gpu_blocks_override:
            n = int(self.cfg.num_gpu_blocks_override)
        elif self.device.type == "cuda":
            free, total = torch.cuda.mem_get_info(self.device)
            used = total - free
            reserve = (3 << 30) + self.runner.max_tokens * (getattr(self.model_cfg, "hidden_size", 4096) * 64)
            budget = total * self.cfg.gpu_memory_utilization - used - reserve - swa_bytes
            min_b = envs.VLLM_B200_MIN_KV_BUDGET_GIB * (1 << 30)
            if budget < min_b:
                raise RuntimeError(f"KV budget {budget / 2**30:.2f} GiB below the minimum "
                                   f"{envs.VLLM_B200_MIN_KV_BUDGET_GIB} GiB; lower max_model_len / max_num_seqs "
                                   "or raise gpu_memory_utilization")
            n = int(budget // per_block)
            if not self.cfg.enable_prefix_caching:
                n = min(n, need)
        else:
            n = need
        if self.world_size > 1:
            n = -self.ps.world.cpu_all_reduce_max([-n])[0]  # min over ranks
        return max(n, 2)

    def initialize_cache(self, num_blocks: int) -> None:
        self.runner.initialize_kv_cache(num_blocks, getattr(self, "num_swa_blocks", 0))

    def warmup(self) -> None:
        t0 = time.time()
        kv = self.cfg.kv_transfer_config
        # a prefill-only server (KV producer) never decodes, so it captures no decode graphs
        # (vllm/worker/neuron_worker.py:957-962); a bucket reached anyway is captured on first use
        producer_only = kv is not None and kv.kv_role == "kv_producer"
        if self.runner.use_graphs and not envs.VLLM_B200_SKIP_DECODE_WARMUP and not producer_only:
            from .scheduler import ScheduledSeq, SchedulerOutput

            for B in self.runner.decode_buckets:
                seqs = [ScheduledSeq(f"__warm{i}", [0], 0, [0], True) for i in range(B)]
                so = SchedulerOutput("decode", seqs)
                # writes go to the reserved null block 0 (never read by a live request)
                self.runner.execute(so)
        buckets = self.cfg.vision_neuron_config.num_vision_tokens_buckets
        if buckets:
            from ..models.interfaces import SupportsVisionWarmup

            if isinstance(self.model, SupportsVisionWarmup):
                # one encoder pass per configured image size, so the first requests do not pay
                # for lazy initialisation (vllm/worker/neuron_worker.py:907 vision warm-up)
                with torch.inference_mode():
                    for b in sorted(set(buckets)):
                        inp = self.model.build_vision_synthetic_inputs(b, self.cfg.vision_neuron_config, self.device)
                        self.model.visual(inp["patches"], inp["grids"])
                self.vision_warmups = len(set(buckets))
        STARTUP_TIME.labels(model_name=self.cfg.served_model_name or str(self.cfg.model)).set(
            time.time() - getattr(self, "_t_start", t0))

    def execute_model(self, so):
        return self.runner.execute(so)

    def shutdown(self) -> None:
        if self.runner is not None:
            self.runner.release_graphs()
        pstate.destroy_parallel_state()
        import torch.distributed as dist

        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:  # noqa: BLE001
                pass
