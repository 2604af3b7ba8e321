"""vLLM worker that runs this framework's engine worker (``parallel_config.worker_cls``).

Counterpart of the Trainium plugin's ``NeuronWorker`` (``vllm_neuron/vllm/worker/neuron_worker.py``)
and its model runner (``neuron_model_runner.py``), which take vLLM's ``SchedulerOutput`` and
return a ``ModelRunnerOutput``.  Here the whole device side is this framework's
(``engine/worker.py``: parallel groups, NVLink / NVLS collectives, model, KV cache, decode
CUDA graphs; ``engine/model_runner.py``: input staging, forward, sampling):

* KV cache: vLLM's KV manager allocates blocks; this worker reports ONE KV-cache "layer"
  whose page is the model's whole per-block footprint (every attention layer's K and V),
  so vLLM's block count equals the number of blocks this framework allocates from the same
  memory budget, and vLLM's block ids index this framework's paged caches directly.
  Prefix-cache hits arrive as ``num_computed_tokens`` > 0 and need nothing else.
* Per-request state: the prompt, the tokens sampled so far (this worker appends every
  token it samples, so a step scheduled before vLLM has processed the previous step's
  output still finds its input token) and the block table (extended by ``new_block_ids``,
  replaced on resumption after preemption).
* Steps: each scheduled request becomes a ``ScheduledSeq`` with the tokens
  ``[num_computed, num_computed + num_scheduled)``; a step of single-token requests that
  all sample is a decode step (graph replay), anything else the varlen path.  A partial
  prefill chunk samples nothing.
* Execution: ``execute_model`` books the step and returns None; ``sample_tokens`` (which
  vLLM calls next, with the grammar bitmask of the step's structured-output requests) runs
  the forward pass and sampling, applying vLLM's packed bitmask (rows of unconstrained
  requests allow every token).

Not routed through this worker: speculative decoding, multimodal inputs, LoRA and pooling
(they run on this framework's own engine, ``vllm-b200 serve``); requests that need them
are refused with an error instead of being served differently.
"""

from __future__ import annotations

import time

import numpy as np
import torch

from ..engine.request import Request
from ..engine.sampling_params import SamplingParams
from ..engine.scheduler import ScheduledSeq, SchedulerOutput
from ..engine.worker import Worker
from ..logging_config import init_logger
from .config_bridge import engine_config_from_vllm

logger = init_logger(__name__)

KV_LAYER_NAME = "b200.kv"


def _sampling(sp) -> SamplingParams:
    """This framework's sampling parameters from vLLM's (temperature / top-k / top-p / seed;
    stop conditions and output limits stay with vLLM's scheduler)."""
    if sp is None:
        return SamplingParams(temperature=0.0, max_tokens=None)
    for name, neutral in (("presence_penalty", 0.0), ("frequency_penalty", 0.0), ("repetition_penalty", 1.0),
                          ("min_p", 0.0)):
        v = getattr(sp, name, neutral)
        if v is not None and float(v) != neutral:
            raise ValueError(f"{name}={v} is not supported by the B200 worker")
    top_k = int(getattr(sp, "top_k", 0) or 0)
    return SamplingParams(temperature=float(sp.temperature), top_p=float(getattr(sp, "top_p", 1.0) or 1.0),
                          top_k=top_k if top_k > 0 else 0, seed=getattr(sp, "seed", None), max_tokens=None)


def _base():
    try:
        from vllm.v1.worker.worker_base import WorkerBase

        return WorkerBase
    except Exception:  # noqa: BLE001 - vLLM absent: a plain base (the class is then unusable by vLLM)
        return object


class B200VllmWorker(_base()):
    def __init__(self, vllm_config, local_rank: int, rank: int, distributed_init_method: str,
                 is_driver_worker: bool = False, device: str = "auto"):
        super().__init__(vllm_config=vllm_config, local_rank=local_rank, rank=rank,
                         distributed_init_method=distributed_init_method, is_driver_worker=is_driver_worker)
        self.cfg = engine_config_from_vllm(vllm_config, device=device)
        self.inner = Worker(self.cfg, rank=rank, world_size=self.cfg.tensor_parallel_size, local_rank=local_rank,
                            init_method=distributed_init_method if self.cfg.tensor_parallel_size > 1 else None)
        self.inner.swa_group_allowed = False  # vLLM keeps one block table per request
        self.requests: dict[str, Request] = {}
        self.block_ids: dict[str, list[int]] = {}
        self._pending: tuple | None = None
        self.steps = 0

    # ------------------------------------------------------------------ set-up
    def init_device(self) -> None:
        self.inner.init_device()
        self.device = self.inner.device

    def load_model(self, *, load_dummy_weights: bool = False) -> None:
        if load_dummy_weights:
            self.cfg.load_format = "dummy"
        self.inner.load_model()

    def get_model(self):
        return self.inner.model

    def page_bytes(self) -> int:
        return max(1, self.inner.model.get_kv_spec().bytes_per_block(self.cfg.block_size))

    def determine_available_memory(self) -> int:
        return self.inner.determine_num_blocks() * self.page_bytes()

    def get_kv_cache_spec(self) -> dict:
        from vllm.v1.kv_cache_interface import FullAttentionSpec

        bs = self.cfg.block_size
        return {KV_LAYER_NAME: FullAttentionSpec(block_size=bs, num_kv_heads=1, head_size=1, dtype=torch.uint8,
                                                 page_size_padded=max(self.page_bytes(), 2 * bs))}

    def get_cache_block_size_bytes(self) -> int:
        return self.page_bytes()

    def initialize_from_config(self, kv_cache_config) -> None:
        self.inner.num_swa_blocks = 0
        self.inner.initialize_cache(int(kv_cache_config.num_blocks))

    def compile_or_warm_up_model(self):
        t0 = time.time()
        self.inner.warmup()
        try:
            from vllm.v1.worker.worker_base import CompilationTimes

            return CompilationTimes(language_model=time.time() - t0, encoder=0.0)
        except ImportError:
            return time.time() - t0

    def get_supported_tasks(self):
        return ("generate",)

    def check_health(self) -> None:
        return None

    def reset_mm_cache(self) -> None:
        return None

    def reset_encoder_cache(self) -> None:
        return None

    def execute_dummy_batch(self) -> None:
        # data-parallel replicas are separate engines here; no cross-replica collective waits
        return None

    def take_draft_token_ids(self):
        return None

    def update_max_model_len(self, max_model_len: int) -> None:
        self.cfg.max_model_len = int(max_model_len)

    def add_lora(self, lora_request) -> bool:
        raise NotImplementedError("LoRA is not supported by the B200 worker")

    def remove_lora(self, lora_id: int) -> bool:
        return False

    def pin_lora(self, lora_id: int) -> bool:
        return False

    def list_loras(self) -> set[int]:
        return set()

    def profile(self, is_start: bool = True, profile_prefix: str | None = None) -> None:
        from ..profiler import Profiler, ProfilerConfig

        if is_start:
            self._profiler = Profiler(ProfilerConfig.from_dict(self.cfg.profiler_config), rank=self.rank)
            self._profiler.start()
        elif getattr(self, "_profiler", None) is not None:
            self._profiler.stop()
            self._profiler = None

    def shutdown(self) -> None:
        self.inner.shutdown()

    # ------------------------------------------------------------------ steps
    def _update_states(self, so) -> None:
        runner = self.inner.runner
        for rid in so.finished_req_ids:
            self.requests.pop(rid, None)
            self.block_ids.pop(rid, None)
            runner.release_state(rid)
        for nr in so.scheduled_new_reqs:
            if getattr(nr, "mm_features", None):
                raise ValueError("multimodal requests are not supported by the B200 worker")
            if getattr(nr, "lora_request", None) is not None:
                raise ValueError("LoRA requests are not supported by the B200 worker")
            if nr.prompt_token_ids is None:
                raise ValueError("prompt embeddings are not supported by the B200 worker")
            req = Request(nr.req_id, list(nr.prompt_token_ids), _sampling(nr.sampling_params))
            req.num_computed_tokens = int(nr.num_computed_tokens)
            self.requests[nr.req_id] = req
            self.block_ids[nr.req_id] = list(nr.block_ids[0])
        cr = so.scheduled_cached_reqs
        for i, rid in enumerate(cr.req_ids):
            req = self.requests[rid]
            new_blocks = cr.new_block_ids[i]
            if rid in cr.resumed_req_ids:
                self.block_ids[rid] = list(new_blocks[0]) if new_blocks is not None else []
            elif new_blocks is not None:
                self.block_ids[rid].extend(new_blocks[0])
            all_ids = cr.all_token_ids.get(rid) if cr.all_token_ids else None
            if all_ids is not None:  # resumed, or not scheduled in the previous step: vLLM's view
                n_prompt = len(req.prompt_token_ids)
                req.output_token_ids = list(all_ids[n_prompt:])
            req.num_computed_tokens = int(cr.num_computed_tokens[i])

    def _schedule(self, so) -> SchedulerOutput:
        if so.scheduled_spec_decode_tokens:
            raise ValueError("speculative decoding through vLLM's scheduler is not supported by the B200 worker")
        seqs = []
        for rid, n in so.num_scheduled_tokens.items():
            req = self.requests[rid]
            start = req.num_computed_tokens
            all_ids = req.all_token_ids
            toks = all_ids[start:start + n]
            if len(toks) != n:
                raise RuntimeError(f"request {rid}: {n} tokens scheduled from position {start}, "
                                   f"{len(all_ids)} known")
            seqs.append(ScheduledSeq(rid, toks, start, self.block_ids[rid], start + n >= len(all_ids),
                                     sampling_params=req.sampling_params, sample_seq=req.sample_seq, request=req))
        kind = "decode" if seqs and all(len(s.token_ids) == 1 and s.sample for s in seqs) else "prefill"
        return SchedulerOutput(kind, seqs)

    def _bitmask(self, ours: SchedulerOutput, grammar) -> torch.Tensor | None:
        """vLLM's packed bitmask (rows in ``structured_output_request_ids`` order) laid out as
        one row per sampled sequence of the step; other rows allow every token."""
        if grammar is None or getattr(grammar, "grammar_bitmask", None) is None:
            return None
        bm = np.asarray(grammar.grammar_bitmask)
        row_of = {rid: i for i, rid in enumerate(grammar.structured_output_request_ids)}
        words = (self.inner.runner.sampler.vocab_size + 31) // 32
        out = np.full((len(ours.seqs), words), -1, dtype=np.int32)
        w = min(words, bm.shape[1])
        for i, s in enumerate(ours.seqs):
            r = row_of.get(s.req_id)
            if r is not None:
                out[i, :w] = bm[r, :w]
                out[i, w:] = 0
        return torch.from_numpy(out)

    def _run(self, so, ours: SchedulerOutput, grammar):
        from vllm.v1.outputs import ModelRunnerOutput

        runner = self.inner.runner
        mask = self._bitmask(ours, grammar)
        if mask is not None:
            runner.external_bitmask = mask
        res = runner.execute(ours) if ours.seqs else {}
        self.steps += 1
        ids, toks = [], []
        for s in ours.seqs:
            t = list(res.get(s.req_id, [])) if s.sample else []
            if t:
                req = self.requests[s.req_id]
                req.output_token_ids.extend(t)
                req.sample_seq += 1
            ids.append(s.req_id)
            toks.append(t)
        return ModelRunnerOutput(req_ids=ids, req_id_to_index={r: i for i, r in enumerate(ids)},
                                 sampled_token_ids=toks)

    @torch.inference_mode()
    def execute_model(self, scheduler_output):
        """Books the step; the forward and sampling run in ``sample_tokens``, which vLLM's
        engine calls next with the grammar bitmask (its batch-queue loop always takes the
        step's output from ``sample_tokens``).  An empty step returns its output here."""
        self._update_states(scheduler_output)
        ours = self._schedule(scheduler_output)
        if not ours.seqs:
            self._pending = None
            return self._run(scheduler_output, ours, None)
        self._pending = (scheduler_output, ours)
        return None

    @torch.inference_mode()
    def sample_tokens(self, grammar_output):
        if self._pending is None:
            from vllm.v1.outputs import EMPTY_MODEL_RUNNER_OUTPUT

            return EMPTY_MODEL_RUNNER_OUTPUT
        so, ours = self._pending
        self._pending = None
        return self._run(so, ours, grammar_output)
