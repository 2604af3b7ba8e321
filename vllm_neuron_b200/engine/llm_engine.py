"""The engine: request intake, scheduling, execution, output assembly.

Multi-GPU execution is SPMD: every rank runs the same scheduler on the same
request stream and therefore issues the same collectives in the same order (the
lockstep invariant the reference protects with its DP MAX-reduce,
``neuron_model_runner.py:2756-2801``).  Three modes:
* ``single``   one rank;
* ``driver``   rank 0 of a multi-process group owns the user API and broadcasts
               new requests / aborts to the followers before every step
               (CPU gloo group);
* ``follower`` ranks 1..N-1 of a driver group, looping on :meth:`step`;
* ``spmd``     every rank is launched externally (torchrun) and receives the same
               requests itself (used by ``bench.py``).
"""

from __future__ import annotations

import os
import time
import uuid
from typing import Any

from ..config import EngineConfig
from ..logging_config import init_logger
from .block_manager import KVCacheManager
from .request import Request, RequestStatus
from .sampling_params import CompletionOutput, RequestOutput, SamplingParams
from .scheduler import Scheduler
from .worker import Worker

logger = init_logger(__name__)


def make_stop_checker(tok, stops: list[str], include: bool):
    """Callable(request) -> True once the decoded output contains a stop string; it sets the
    request's ``stop_reason`` (the string) and ``stop_text`` (the output cut before it, or after
    it with ``include``).  Only the new tail of the text is searched each step."""
    longest = max(len(x) for x in stops)

    def check(req) -> bool:
        text = tok.decode(req.output_token_ids, skip_special_tokens=True)
        start = max(0, getattr(req, "_stop_scanned", 0) - longest)
        req._stop_scanned = len(text)
        hits = [(text.find(x, start), x) for x in stops]
        hits = [(p, x) for p, x in hits if p >= 0]
        if not hits:
            return False
        p, x = min(hits)
        req.stop_reason = x
        req.stop_text = text[:p + (len(x) if include else 0)]
        return True

    return check


class LLMEngine:
    def __init__(self, cfg: EngineConfig, rank: int = 0, world_size: int = 1, local_rank: int = 0,
                 mode: str = "single"):
        self.cfg = cfg
        self.rank, self.world_size, self.mode = rank, world_size, mode
        self.worker = Worker(cfg, rank, world_size, local_rank)
        self.worker.init_device()
        self.worker.load_model()
        n_blocks = self.worker.determine_num_blocks()
        self.worker.initialize_cache(n_blocks)
        self.proposer = None
        if cfg.speculative_config is not None and cfg.data_parallel_size > 1:
            raise ValueError("speculative decoding with data_parallel_size > 1 is not supported")
        if cfg.speculative_config is not None:
            from ..spec_decode.eagle import EagleProposer

            # verification steps carry k+1 tokens per request and run eagerly
            self.worker.runner.use_graphs = False
            self.proposer = EagleProposer(cfg, self.worker)
        self.worker.warmup()
        self.num_blocks = n_blocks
        hybrid = hasattr(self.worker.model, "get_state_spec")
        if hybrid and cfg.enable_prefix_caching:
            logger.info("prefix caching disabled: recurrent (linear-attention) layers keep per-request state")
        # with decode context parallelism a block-table entry covers block_size tokens on each
        # of the dcp ranks
        n_swa = getattr(self.worker, "num_swa_blocks", 0)
        self.kv = KVCacheManager(n_blocks, cfg.block_size * cfg.decode_context_parallel_size,
                                 cfg.enable_prefix_caching and not hybrid,
                                 sliding_window=self.worker.swa_group_window() if n_swa else None, swa_blocks=n_swa)
        if n_swa:
            logger.info("sliding-window layers use their own KV group: %d blocks (full-attention layers: %d)",
                        n_swa, n_blocks)
        k = cfg.speculative_config.num_speculative_tokens if cfg.speculative_config else 0
        # mixed prefill + decode steps need no lockstep step kinds (data parallelism), no
        # speculation and no context-parallel attention
        mixed = cfg.mixed_prefill_tokens if (cfg.data_parallel_size == 1 and k == 0
                                             and cfg.decode_context_parallel_size == 1) else 0
        self.scheduler = Scheduler(self.kv, cfg.max_num_seqs, cfg.max_num_batched_tokens, cfg.max_model_len,
                                   cfg.max_num_prefills_per_step, cfg.enable_chunked_prefill, k,
                                   mixed_prefill_tokens=mixed)
        if self.worker.runner.encoder_cache is not None:
            self.scheduler.on_finish.append(self.worker.runner.encoder_cache.release)
        if self.worker.runner.debug_logits is not None:
            self.worker.runner.debug_logits.replica = rank // cfg.tensor_parallel_size
            self.scheduler.on_finish.append(self.worker.runner.debug_logits.release)
        if self.worker.runner.state_caches is not None:
            self.scheduler.on_finish.append(self.worker.runner.release_state)
            self.scheduler.on_preempt.append(self.worker.runner.release_state)
        hf = self.worker.hf
        self.eos_token_id = hf.get("eos_token_id")
        from ..profiler import Profiler, ProfilerConfig

        self.profiler = Profiler(ProfilerConfig.from_dict(cfg.profiler_config), rank)
        self.connector = None
        if cfg.kv_transfer_config is not None:
            if cfg.decode_context_parallel_size > 1:
                raise ValueError("KV transfer with decode context parallelism is not supported")
            self._init_connector(hf)
        self._pending: list[tuple] = []
        self._stopped = False
        # data parallelism: requests are dealt round-robin to replicas (same order on every
        # rank); outputs are exchanged over the DP group every step
        self.dp = cfg.data_parallel_size
        self.replica = rank // cfg.tensor_parallel_size
        self._rr = 0
        self._dp_step = 0  # data-parallel lockstep counter (checked every step)
        self._remote: set[str] = set()  # unfinished requests owned by other replicas
        # asynchronous scheduling (single rank or SPMD; decode steps with CUDA graphs)
        # (grammar masks need step k's token before step k + 1 is staged: no lookahead then)
        self._async = bool(cfg.async_scheduling) and self.dp == 1 and mode in ("single", "spmd") \
            and not cfg.neuron_config.enable_structured_outputs \
            and self.proposer is None
        self._inflight = None
        self.async_stats = {"launched": 0, "lookahead": 0, "sync_fallback": 0}
        logger.info("engine ready: rank %d/%d mode=%s kv_blocks=%d", rank, world_size, mode, n_blocks)

    # ------------------------------------------------------------------ intake
    def add_request(self, request_id: str | None, prompt_token_ids: list[int], sampling_params: SamplingParams,
                    prompt: str | None = None, mm_inputs: list | None = None,
                    kv_transfer_params: dict | None = None) -> str:
        rid = request_id or uuid.uuid4().hex
        req = self._make_request(rid, prompt_token_ids, sampling_params, prompt, mm_inputs, kv_transfer_params)
        if self.mode == "driver":
            self._pending.append(("add", rid, req.prompt_token_ids, sampling_params, prompt, mm_inputs,
                                  kv_transfer_params))
        self._admit(req)
        return rid

    def _admit(self, req: Request) -> None:
        owner = self._rr
        self._rr = (self._rr + 1) % self.dp
        if owner == self.replica:
            self.scheduler.add_request(req)
        else:
            self._remote.add(req.request_id)

    def structured_output_manager(self):
        """Grammar compiler over this model's vocabulary (built on the first constrained
        request from the model's tokenizer, or set by the caller as ``so_manager``).
        Constrained requests are refused unless ``enable_structured_outputs`` is on, as in the
        reference (``vllm/platform.py:396-435``)."""
        if not self.cfg.neuron_config.enable_structured_outputs:
            raise ValueError("structured outputs are disabled: set neuron_config.enable_structured_outputs")
        if self.cfg.speculative_config is not None:
            raise ValueError("structured outputs with speculative decoding are not supported")
        if getattr(self, "so_manager", None) is None:
            from .structured_output import StructuredOutputManager

            vocab = getattr(self.worker.model_cfg, "vocab_size", None) or self.worker.hf.get("vocab_size")
            self.so_manager = StructuredOutputManager.from_tokenizer(self.tokenizer(), vocab)
        return self.so_manager

    def tokenizer(self):
        """The model directory's tokenizer (loaded on first use: stop strings, structured
        outputs); a caller may set ``engine.hf_tokenizer`` instead."""
        if getattr(self, "hf_tokenizer", None) is None:
            from transformers import AutoTokenizer

            if self.cfg.model is None:
                raise ValueError("stop strings / structured outputs need a tokenizer: load a model directory")
            self.hf_tokenizer = AutoTokenizer.from_pretrained(self.cfg.model)
        return self.hf_tokenizer

    def max_embeds_per_image(self) -> int | None:
        """Largest image (in merged vision tokens) a request may carry: the largest
        ``num_vision_tokens_buckets`` entry when buckets are configured, else what the whole
        encoder cache holds.  None for text-only models."""
        ec = getattr(self.worker.runner, "encoder_cache", None)
        if ec is None:
            return None
        cap = ec.buf.shape[0] * ec.block_size
        buckets = self.cfg.vision_neuron_config.num_vision_tokens_buckets
        return min(cap, max(buckets)) if buckets else cap

    def _make_request(self, rid, prompt_token_ids, sampling_params, prompt, mm_inputs, kv_transfer_params) -> Request:
        ids = list(map(int, prompt_token_ids))
        req = Request(rid, ids, sampling_params, self.eos_token_id, prompt, mm_inputs=mm_inputs,
                      kv_transfer_params=kv_transfer_params)
        n_lp = sampling_params.logprobs
        if n_lp is not None:
            limit = self.cfg.neuron_config.max_logprobs or 20
            if n_lp < 0 or n_lp > limit:
                raise ValueError(f"logprobs must be in [0, {limit}] (neuron_config.max_logprobs)")
            if self.proposer is not None:
                raise ValueError("logprobs with speculative decoding are not supported")
        so = getattr(sampling_params, "structured_outputs", None)
        if so is not None:
            req.grammar = self.structured_output_manager().matcher(so)
        if sampling_params.stop:
            req.stop_checker = make_stop_checker(self.tokenizer(), sampling_params.stop,
                                                 sampling_params.include_stop_str_in_output)
        model = self.worker.model
        if mm_inputs and hasattr(model, "embed_multimodal"):
            from ..models.qwen3_vl import preprocess_image

            images = []
            for item in mm_inputs:
                img = item.get("image") if isinstance(item, dict) else item
                if img is None:
                    continue
                images += list(img) if isinstance(img, (list, tuple)) else [img]
            img_tok = model.vl_cfg.image_token_id
            grids = [preprocess_image(torch_image(im), model.vl_cfg.vision)[1] for im in images]
            counts = [model.num_image_tokens(g) for g in grids]
            cap = self.max_embeds_per_image()
            for n in counts:
                if cap is not None and n > cap:
                    # refused before scheduling, so an oversized image never reaches the encoder
                    # cache mid-step (vllm_neuron/vllm/platform.py:396 validate_request)
                    raise ValueError(f"an image in this request produces {n} embedding tokens, which exceeds the "
                                     f"maximum of the vision encoder cache ({cap}); reduce the image resolution "
                                     f"or raise vision_neuron_config.max_vision_seq_len / num_vision_tokens_buckets")
            n_ph = sum(1 for t in ids if t == img_tok)
            out, items, gi, i = [], [], 0, 0
            if n_ph == len(grids):  # one placeholder per image: expand each to its token count
                for t in ids:
                    if t == img_tok:
                        items.append({"pixels": torch_image(images[gi]), "grid": grids[gi], "offset": len(out),
                                      "n": counts[gi]})
                        out += [img_tok] * counts[gi]
                        gi += 1
                    else:
                        out.append(t)
            elif n_ph == sum(counts):  # already expanded: record where each image starts
                out = list(ids)
                while i < len(out):
                    if out[i] == img_tok:
                        items.append({"pixels": torch_image(images[gi]), "grid": grids[gi], "offset": i,
                                      "n": counts[gi]})
                        i += counts[gi]
                        gi += 1
                    else:
                        i += 1
            else:
                raise ValueError(f"prompt has {n_ph} image tokens for {len(grids)} images ({sum(counts)} tokens)")
            req.prompt_token_ids = out
            req.mm_items = items
            req.mrope_positions, req.mrope_delta = model.mrope_positions(out, grids)
        return req

    def _init_connector(self, hf: dict) -> None:
        from ..kv_transfer import make_connector
        from ..models.base import kv_head_sharding

        extra = self.cfg.kv_transfer_config.kv_connector_extra_config
        if not extra.get("engine_id"):
            eid = uuid.uuid4().hex[:12]
            if self.world_size > 1:  # every rank of this engine names its transfers alike
                eid = self.worker.ps.world.broadcast_object(eid)
            extra["engine_id"] = eid
        tp = self.worker.ps.tp
        n_kv = hf.get("num_key_value_heads") or hf.get("num_attention_heads") or 1
        rng = kv_head_sharding(n_kv, tp.world_size, tp.rank_in_group)
        self.connector = make_connector(self.cfg, self.worker.runner, tp.rank_in_group, tp.world_size, rng)
        self.scheduler.connector = self.connector

    def start_profile(self) -> None:
        if self.mode == "driver":
            self._pending.append(("profile", True))
        self.profiler.start()

    def stop_profile(self) -> dict:
        if self.mode == "driver":
            self._pending.append(("profile", False))
        return self.profiler.stop()

    def abort_request(self, request_id: str) -> None:
        self._remote.discard(request_id)
        if self.mode == "driver":
            self._pending.append(("abort", request_id))
        self.scheduler.abort(request_id)

    def has_unfinished_requests(self) -> bool:
        return self.scheduler.has_unfinished() or bool(self._remote) or self._inflight is not None

    # -------------------------------------------------------------------- step
    def _sync_requests(self) -> None:
        if self.mode not in ("driver", "follower"):
            return
        msgs = self.worker.ps.world.broadcast_object(self._pending if self.rank == 0 else None)
        self._pending = []
        if self.mode == "follower":
            for m in msgs:
                if m[0] == "add":
                    _, rid, ids, sp, prompt, mm, kvp = m
                    self._admit(self._make_request(rid, ids, sp, prompt, mm, kvp))
                elif m[0] == "abort":
                    self.scheduler.abort(m[1])
                elif m[0] == "profile":
                    if m[1]:
                        self.profiler.start()
                    else:
                        self.profiler.stop()
                elif m[0] == "shutdown":
                    self._stopped = True

    def step(self) -> list[RequestOutput]:
        self.profiler.step()
        self._sync_requests()
        if self._stopped:
            return []
        if self.dp > 1:
            return self._step_dp()
        if self._async:
            return self._step_async()
        so = self.scheduler.schedule()
        failed = [self._make_output(r, True) for r in self.scheduler.failed]
        self.scheduler.failed = []
        if so.kind == "idle":
            return failed
        return failed + self._run(so)

    def _step_async(self) -> list[RequestOutput]:
        """Asynchronous scheduling (``async_scheduling=True``): while decode step k runs on
        the GPU, the host schedules and stages step k+1 (its input tokens are step k's sampled
        ids, taken on the device) and only then waits for step k's ids, appends them and
        checks stop conditions; outputs therefore trail the GPU by one step.  Anything else
        (prefill, preemption, a request at its last token) drains the pipeline first and runs
        synchronously."""
        runner, sched = self.worker.runner, self.scheduler
        prev = self._inflight
        if prev is not None:
            nxt = sched.schedule_lookahead()
            cur = None
            if nxt is not None:
                cur = runner.launch(nxt, prev)
                self._count_async("lookahead")
                self._mark_inflight(nxt, 1)
            outs = self._commit(prev)
            self._inflight = cur
            return outs
        so = sched.schedule()
        failed = [self._make_output(r, True) for r in sched.failed]
        sched.failed = []
        if so.kind == "idle":
            return failed
        if runner.can_launch_async(so):
            self._inflight = runner.launch(so)
            self._count_async("launched")
            self._mark_inflight(so, 1)
            return failed
        self._count_async("sync_fallback")
        return failed + self._run(so)

    def _count_async(self, mode: str) -> None:
        """Async vs synchronous-fallback step counters (reference:
        ``neuron_model_runner.py:709-710``, ``neuron_worker.py:1881-1897``)."""
        from ..metrics import ASYNC_STEPS

        self.async_stats[mode] += 1
        ASYNC_STEPS.labels(model_name=self.cfg.served_model_name or "model", mode=mode).inc()

    @staticmethod
    def _mark_inflight(so, sign: int) -> None:
        """Launched (+1) or committed (-1): decode tokens count in num_inflight, prompt chunks
        of mixed steps in num_inflight_prefill."""
        for i, s in enumerate(so.seqs):
            if so.kind == "mixed" and i >= so.num_decode:
                s.request.num_inflight_prefill += sign * len(s.token_ids)
            else:
                s.request.num_inflight += sign

    def _commit(self, step) -> list[RequestOutput]:
        sampled = self.worker.runner.commit(step)
        self._mark_inflight(step.so, -1)
        finished = self.scheduler.update_from_output(step.so, sampled, time.monotonic())
        fin = {r.request_id for r in finished}
        return [self._make_output(s.request, s.request.status.finished) for s in step.so.seqs
                if s.req_id in sampled and (s.req_id in fin or not s.request.status.finished)]

    def _step_dp(self) -> list[RequestOutput]:
        """One lockstep step of a data-parallel replica.  Replicas share the MoE layers'
        collectives, so every replica runs a step of the same kind with the same padded
        token count (idle replicas run a padding batch), the counterpart of the reference's
        per-step MAX-reduce and dummy batches (``neuron_model_runner.py:6524-6821,6968``)."""
        world = self.worker.ps.world
        self._dp_step += 1
        has_work = self.scheduler.has_unfinished()
        flags = world.lockstep_all_reduce_max([int(has_work), int(has_work and self.scheduler.has_prefill_work())],
                                              self._dp_step, 1)
        outs: list[RequestOutput] = []
        if flags[0]:
            kind = "prefill" if flags[1] else "decode"
            so = self.scheduler.schedule(kind)
            outs = [self._make_output(r, True) for r in self.scheduler.failed]
            self.scheduler.failed = []
            n_tok = so.num_tokens if so.kind != "idle" else 0
            mx = world.lockstep_all_reduce_max([n_tok, len(so.seqs)], self._dp_step, 2)
            outs += self._run(so, dp_pad=(kind, mx[0], mx[1]))
        # every replica learns every replica's outputs (TP peers hold identical copies)
        allouts = [o for lst in self.worker.ps.dp.all_gather_object(outs) for o in lst]
        for o in allouts:
            if o.finished:
                self._remote.discard(o.request_id)
        return allouts

    def _run(self, so, dp_pad=None) -> list[RequestOutput]:
        if so.kind == "idle":  # data-parallel padding step
            self.worker.runner.execute(so, dp_pad=dp_pad)
            return []
        if self.proposer is not None and so.kind == "decode":
            sampled = self.proposer.execute_with_speculation(so)
        else:
            sampled = self.worker.runner.execute(so, dp_pad=dp_pad) if dp_pad else self.worker.execute_model(so)
            for rid, entry in getattr(self.worker.runner, "last_logprobs", {}).items():
                req = self.scheduler.requests.get(rid)
                if req is not None:
                    req.logprobs.append(entry)
        now = time.monotonic()
        finished = self.scheduler.update_from_output(so, sampled, now)
        if self.proposer is not None:
            self.proposer.propose(so, sampled, self.scheduler)
        outs = []
        fin_ids = {r.request_id for r in finished}
        for s in so.seqs:
            if s.req_id in sampled or s.req_id in fin_ids:
                req = s.request
                outs.append(self._make_output(req, req.status.finished))
        return outs

    def _make_output(self, req: Request, finished: bool) -> RequestOutput:
        reason = None
        if req.status == RequestStatus.FINISHED_STOPPED:
            reason = "stop"
        elif req.status == RequestStatus.FINISHED_LENGTH:
            reason = "length"
        elif req.status == RequestStatus.FINISHED_ABORTED:
            reason = "abort"
        return RequestOutput(req.request_id, req.prompt, req.prompt_token_ids,
                             [CompletionOutput(0, req.stop_text or "", list(req.output_token_ids), reason,
                                               list(req.logprobs) if req.sampling_params.logprobs is not None
                                               else None, req.stop_reason)], finished,
                             req.metrics, req.num_cached_tokens, req.kv_transfer_params_out)

    # ------------------------------------------------------------------ scoring
    def score(self, prompt_token_ids: list[int]) -> "torch.Tensor":
        """Logits [len(prompt), vocab] of a prompt (teacher forcing), for accuracy tools.
        Single-rank and SPMD engines only (every rank must call it)."""
        import torch  # noqa: F401

        from .scheduler import ScheduledSeq, SchedulerOutput

        if self.mode in ("driver", "follower"):
            raise RuntimeError("score() needs a single-rank or SPMD engine")
        if self.scheduler.has_unfinished():
            raise RuntimeError("score() needs an idle engine")
        ids = list(map(int, prompt_token_ids))
        req = Request(f"__score_{uuid.uuid4().hex}", ids, SamplingParams(max_tokens=1))
        if not self.kv.allocate_slots(req, len(ids)):
            raise RuntimeError("not enough KV blocks to score the prompt")
        try:
            seq = ScheduledSeq(req.request_id, ids, 0, list(req.block_ids), False, request=req)
            vocab = getattr(self.worker.model_cfg, "vocab_size", None) or self.worker.hf["vocab_size"]
            return self.worker.runner.score(SchedulerOutput("prefill", [seq]), vocab)
        finally:
            self.kv.free(req)
            if self.worker.runner.state_caches is not None:
                self.worker.runner.release_state(req.request_id)

    # ---------------------------------------------------------------- lifecycle
    def run_follower(self) -> None:
        while not self._stopped:
            self.step()

    def shutdown(self) -> None:
        if self.mode == "driver" and not self._stopped:
            self._pending.append(("shutdown",))
            self._sync_requests()
        self._stopped = True
        if self.connector is not None:
            self.connector.cleanup()
        self.worker.shutdown()

    # -------------------------------------------------------------- statistics
    def stats(self) -> dict[str, Any]:
        return {"kv_usage": self.kv.usage, "num_blocks": self.num_blocks,
                "running": len(self.scheduler.running), "waiting": len(self.scheduler.waiting),
                "h2d_bytes_last": self.worker.runner.h2d_bytes_last,
                "d2h_bytes_last": self.worker.runner.d2h_bytes_last}


def torch_image(x):
    """Accept a CHW tensor / HWC numpy array / PIL image; return a CHW float tensor."""
    import numpy as np
    import torch

    if isinstance(x, torch.Tensor):
        t = x.float()
    else:
        arr = np.asarray(x)
        t = torch.from_numpy(arr.copy()).float()
        if t.dim() == 3 and t.shape[-1] in (1, 3, 4):
            t = t.permute(2, 0, 1)
    if t.dim() == 3 and t.shape[0] == 4:
        t = t[:3]
    return t


def _follower_main(cfg: EngineConfig, rank: int, world_size: int, master_port: int = 0) -> None:
    """Entry of a follower rank spawned by ``LLM`` (rendezvous through the file store
    named in the environment; ``master_port`` only for TCP rendezvous)."""
    if master_port:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(master_port)
    eng = LLMEngine(cfg, rank, world_size, local_rank=rank, mode="follower")
    try:
        eng.run_follower()
    finally:
        eng.worker.shutdown()
