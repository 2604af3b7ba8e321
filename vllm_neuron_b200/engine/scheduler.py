"""Continuous-batching scheduler.

Policy (restated from the Trainium plugin's ``NeuronScheduler``,
``vllm_neuron/vllm/core/scheduler.py:78-906``):
* a step is either all-prefill or all-decode; while a prefill is pending the decode
  requests are held back (``scheduler.py:821-854``);
* at most ``max_num_prefills_per_step`` prompts per prefill step (the reference fixes
  it at 1, ``:201``; the default here is the same);
* long prompts are prefilled in segments of at most ``max_num_batched_tokens``
  (segmented prefill), earlier segments land in the paged cache and later ones
  attend to them;
* KV admission control: no new prompt is admitted while the running set could,
  at worst-case length ``max_model_len``, exhaust the cache (``:556-580``), so decode
  never preempts decode in steady state; if it still runs out of blocks the newest
  running request is preempted and recomputed later;
* decode batches are padded to the ``num_seqs_buckets`` graph sizes by the runner;
  the padding is recorded in the ``num_seqs_padding`` histogram.

Every rank runs this scheduler on the same inputs and reaches the same decisions,
which keeps the ranks' collectives in lockstep without broadcasting schedules.
"""

from __future__ import annotations

import time
from collections import deque
from dataclasses import dataclass, field

from ..logging_config import init_logger
from .block_manager import KVCacheManager
from .request import Request, RequestStatus

logger = init_logger(__name__)


def token_hash(tokens) -> str:
    """Fingerprint of a token sequence carried with a KV transfer, so the receiver can check
    that the KV belongs to its prompt's prefix."""
    import hashlib

    import numpy as np

    return hashlib.sha1(np.asarray(list(tokens), dtype=np.int64).tobytes()).hexdigest()


@dataclass
class ScheduledSeq:
    req_id: str
    token_ids: list[int]  # tokens whose K/V are computed this step
    start_pos: int  # position of token_ids[0]
    block_ids: list[int]
    sample: bool  # sample a token after this step
    spec_token_ids: list[int] = field(default_factory=list)
    sampling_params: object = None
    sample_seq: int = 0
    mm_inputs: list | None = None
    request: Request | None = None
    swa_block_ids: list[int] | None = None  # the windowed layers' table (separate KV group)

    @property
    def seq_len(self) -> int:
        return self.start_pos + len(self.token_ids)


@dataclass
class SchedulerOutput:
    kind: str  # "prefill" | "decode" | "mixed" | "idle"
    seqs: list[ScheduledSeq]
    preempted: list[str] = field(default_factory=list)
    finished: list[str] = field(default_factory=list)
    # "mixed": the first num_decode seqs are single-token decodes, the rest prefill chunks
    num_decode: int = 0

    @property
    def num_tokens(self) -> int:
        return sum(len(s.token_ids) for s in self.seqs)


class Scheduler:
    def __init__(self, kv: KVCacheManager, max_num_seqs: int, max_num_batched_tokens: int, max_model_len: int,
                 max_num_prefills_per_step: int = 1, enable_chunked_prefill: bool = True,
                 num_spec_tokens: int = 0, mixed_prefill_tokens: int = 0):
        self.kv = kv
        # > 0: while requests are decoding, prompt work rides along in their steps, at most this
        # many prompt tokens per step (a decode step streams every expert weight anyway, so a
        # prompt chunk adds little); 0: prefill and decode run as separate steps
        self.mixed_prefill_tokens = mixed_prefill_tokens
        self.max_num_seqs = max_num_seqs
        self.max_num_batched_tokens = max_num_batched_tokens
        self.max_model_len = max_model_len
        self.max_prefills = max_num_prefills_per_step
        self.chunked = enable_chunked_prefill
        self.num_spec_tokens = num_spec_tokens
        self.waiting: deque[Request] = deque()
        self.running: list[Request] = []
        self.requests: dict[str, Request] = {}
        blocks_per_max = -(-max_model_len // kv.block_size)
        self.max_kv_concurrent = max(1, (kv.pool.num_blocks - 1) // blocks_per_max)
        self._finished_ids: list[str] = []
        self.on_finish: list = []  # callbacks(request_id), e.g. encoder-cache release
        self.on_preempt: list = []  # callbacks(request_id), e.g. recurrent-state slot release
        self.connector = None  # KV-transfer connector (disaggregated prefill / decode)
        # decode -> prefill KV for multi-turn chats (VLLM_B200_BIDIRECTIONAL_KV)
        from .. import envs

        self.bidirectional_kv = bool(envs.VLLM_B200_BIDIRECTIONAL_KV)
        self.failed: list[Request] = []  # aborted at admission; the engine reports them

    # ------------------------------------------------------------------ queue
    def add_request(self, req: Request) -> None:
        if req.num_prompt_tokens >= self.max_model_len:
            raise ValueError(f"prompt of {req.num_prompt_tokens} tokens exceeds max_model_len {self.max_model_len}")
        if req.num_prompt_tokens == 0:
            raise ValueError("empty prompt")
        self.requests[req.request_id] = req
        self.waiting.append(req)

    def abort(self, req_id: str) -> None:
        req = self.requests.get(req_id)
        if req is None or req.status.finished:
            return
        req.status = RequestStatus.FINISHED_ABORTED
        self._finish(req)

    def has_unfinished(self) -> bool:
        return bool(self.waiting or self.running)

    def _finish(self, req: Request) -> None:
        c = self.connector
        p = req.kv_transfer_params or {}
        ok = req.status != RequestStatus.FINISHED_ABORTED and bool(req.block_ids)
        if c is not None and c.is_producer and p.get("do_remote_decode") and ok:
            # hand the prompt KV to the decode engine before the blocks are freed
            req.kv_transfer_params_out = c.export(req.request_id, req.block_ids, req.num_prompt_tokens)
            req.kv_transfer_params_out["token_hash"] = token_hash(req.prompt_token_ids)
        elif (c is not None and c.is_consumer and p.get("do_remote_prefill") and p.get("return_kv") and ok
              and self.bidirectional_kv and req.num_computed_tokens > 0):
            # bidirectional KV (decode -> prefill): the conversation so far (prompt and output,
            # every token whose KV is written) goes back, so the next turn's prefill engine loads
            # it instead of recomputing it.  Only requests that ask for it (``return_kv``: the
            # client expects another turn) pay for the export, which copies every layer's KV of
            # the conversation (device pool, or device -> host + a file when the pool is absent
            # or full) on the scheduler thread; the export expires after the connector's
            # ``return_ttl_s`` (60 s by default) instead of its ``ttl_s``.
            n = req.num_computed_tokens
            out = c.export(req.request_id + "-d2p", req.block_ids, n, ttl_s=getattr(c, "return_ttl_s", None))
            out["token_hash"] = token_hash((list(req.prompt_token_ids) + list(req.output_token_ids))[:n])
            req.kv_transfer_params_out = out
        for cb in self.on_finish:
            cb(req.request_id)
        if req in self.running:
            self.running.remove(req)
        try:
            self.waiting.remove(req)
        except ValueError:
            pass
        self.kv.free(req)
        req.metrics.finished_time = time.monotonic()
        self._finished_ids.append(req.request_id)
        self.requests.pop(req.request_id, None)

    # --------------------------------------------------------------- schedule
    def _is_prefill(self, r: Request) -> bool:
        return r.num_computed_tokens < r.num_prompt_tokens

    def can_admit(self) -> bool:
        """Room for one more sequence (batch size and worst-case KV capacity).  Whether a
        segmented prefill from an earlier step is still in flight is checked by the caller."""
        if len(self.running) >= self.max_num_seqs:
            return False
        return len(self.running) < self.max_kv_concurrent

    def has_prefill_work(self) -> bool:
        """A prefill step would do something now (a segment in flight or an admissible prompt)."""
        if any(self._is_prefill(r) for r in self.running):
            return True
        return bool(self.waiting) and self.can_admit()

    def schedule(self, kind: str | None = None) -> SchedulerOutput:
        """Next step.  ``kind`` ("prefill" | "decode") restricts the step type; data-parallel
        replicas use it to run the same kind of step in lockstep (a replica with nothing of
        that kind gets an idle output and runs a padding batch).  With ``mixed_prefill_tokens``
        a step that has both decoding requests and prompt work is one "mixed" step."""
        if kind is None and self.mixed_prefill_tokens > 0 and not self.num_spec_tokens:
            decoders = [r for r in self.running if not self._is_prefill(r)]
            if decoders and self.has_prefill_work():
                return self._schedule_mixed(decoders)
        finished, self._finished_ids = self._finished_ids, []
        # 1) ongoing segmented prefills first
        pre = [r for r in self.running if self._is_prefill(r)] if kind != "decode" else []
        # 2) admit new prompts when no prefill is in flight
        if not pre and kind != "decode":
            admitted = 0
            while self.waiting and admitted < self.max_prefills and self.can_admit():
                req = self.waiting[0]
                remote = self._remote_prefill_tokens(req)
                if remote > 0:
                    # disaggregated decode: the prompt KV (all but the last token) comes from the
                    # prefill engine; this engine computes only the last prompt token
                    req.num_computed_tokens = 0
                    if not self.kv.allocate_slots(req, req.num_prompt_tokens):
                        break
                    try:
                        self.connector.load(req.kv_transfer_params, req.block_ids, remote)
                    except Exception as e:  # noqa: BLE001  (missing / malformed transfer)
                        logger.error("request %s: KV transfer failed: %s", req.request_id, e)
                        self.waiting.popleft()
                        req.status = RequestStatus.FINISHED_ABORTED
                        self._finish(req)
                        self.failed.append(req)
                        continue
                    req.num_computed_tokens = remote
                    req.num_cached_tokens = remote
                else:
                    blocks, n_cached = self.kv.get_computed_blocks(req)
                    req.num_computed_tokens = n_cached
                    req.num_cached_tokens = n_cached
                    n_new = self._prefill_chunk(req)
                    if not self.kv.allocate_slots(req, n_new, blocks):
                        req.num_computed_tokens = 0
                        break
                self.waiting.popleft()
                req.status = RequestStatus.RUNNING
                if req.metrics.first_scheduled_time is None:
                    req.metrics.first_scheduled_time = time.monotonic()
                self.running.append(req)
                pre.append(req)
                admitted += 1
                if self._budget_left(pre) <= 0:
                    break
        if pre:
            seqs = []
            budget = self.max_num_batched_tokens
            for req in pre:
                if budget <= 0:
                    break
                n = min(self._prefill_chunk(req), budget)
                if not self.kv.allocate_slots(req, n):
                    break
                budget -= n
                s = req.num_computed_tokens
                done = s + n >= req.num_tokens
                seqs.append(ScheduledSeq(req.request_id, req.all_token_ids[s:s + n], s, req.block_ids, done,
                                         sampling_params=req.sampling_params, sample_seq=req.sample_seq,
                                         mm_inputs=req.mm_inputs, request=req, swa_block_ids=self._swa(req)))
            if seqs:
                return SchedulerOutput("prefill", seqs, finished=finished)
        if kind == "prefill":
            return SchedulerOutput("idle", [], [], finished)
        # 3) decode step over every running request
        seqs, preempted = self._decode_seqs(list(self.running))
        if not seqs:
            return SchedulerOutput("idle", [], preempted, finished)
        return SchedulerOutput("decode", seqs, preempted, finished)

    def _schedule_mixed(self, decoders: list[Request]) -> SchedulerOutput:
        """Every decoding request (one token each; their KV slots are secured first, preempting
        the newest if needed) followed by prompt chunks within ``mixed_prefill_tokens``."""
        finished, self._finished_ids = self._finished_ids, []
        dec, preempted = self._decode_seqs(decoders)
        saved = self.max_num_batched_tokens
        self.max_num_batched_tokens = self.mixed_prefill_tokens
        try:
            pre = self.schedule("prefill")
        finally:
            self.max_num_batched_tokens = saved
        seqs = dec + (pre.seqs if pre.kind == "prefill" else [])
        if not seqs:
            return SchedulerOutput("idle", [], preempted, finished)
        if not dec:
            return SchedulerOutput("prefill", seqs, preempted, finished)
        if len(seqs) == len(dec):
            return SchedulerOutput("decode", seqs, preempted, finished)
        return SchedulerOutput("mixed", seqs, preempted, finished, num_decode=len(dec))

    def _decode_seqs(self, running: list[Request]) -> tuple[list[ScheduledSeq], list[str]]:
        seqs, preempted = [], []
        k = self.num_spec_tokens
        i = 0
        while i < len(running):
            req = running[i]
            n_new = 1 + len(req.spec_token_ids[:k])
            if not self.kv.allocate_slots(req, n_new):
                # preempt the newest request and retry
                victim = running.pop()
                self._preempt(victim)
                preempted.append(victim.request_id)
                if victim is req:
                    continue
                continue
            i += 1
        for req in running:
            spec = req.spec_token_ids[:k]
            s = req.num_computed_tokens
            toks = [req.token_at(s)] + spec if s < req.num_tokens else spec
            seqs.append(ScheduledSeq(req.request_id, toks, s, req.block_ids, True, spec_token_ids=spec,
                                     sampling_params=req.sampling_params, sample_seq=req.sample_seq, request=req,
                                     swa_block_ids=self._swa(req)))
        return seqs, preempted

    def schedule_lookahead(self) -> SchedulerOutput | None:
        """Asynchronous scheduling: the next step while the previous one is still on the GPU.
        Every decoding request feeds the token that the in-flight step is sampling (the runner
        takes it from device memory), at position num_computed + num_inflight.  With mixed
        steps, a prompt whose chunk is in flight continues with its next chunk (its tokens are
        known on the host).  Returns None when that is not possible (a prompt to admit, a
        prompt whose last chunk is in flight, speculation, a request at its token limit, no
        free KV block): the caller then drains the pipeline."""
        if self.num_spec_tokens or not self.running:
            return None
        mixed = self.mixed_prefill_tokens > 0
        if self.waiting and (not mixed or self.can_admit()):
            return None
        dec, pre = [], []
        budget = self.mixed_prefill_tokens
        for req in self.running:
            if self._is_prefill(req):
                start = req.num_computed_tokens + req.num_inflight_prefill
                if not mixed or req.num_inflight or start >= req.num_prompt_tokens:
                    return None  # no chunk in flight yet, or the last one is: decide after it lands
                n = min(req.num_prompt_tokens - start, budget)
                if n <= 0:
                    continue
                if not self.kv.allocate_slots(req, req.num_inflight_prefill + n):
                    return None
                budget -= n
                pre.append(ScheduledSeq(req.request_id, req.prompt_token_ids[start:start + n], start,
                                        req.block_ids, start + n >= req.num_tokens,
                                        sampling_params=req.sampling_params, sample_seq=req.sample_seq,
                                        mm_inputs=req.mm_inputs, request=req, swa_block_ids=self._swa(req)))
                continue
            if req.num_inflight != 1:
                return None
            if len(req.output_token_ids) + 1 >= req.max_tokens:
                return None  # the in-flight token ends this request: nothing to run ahead
            if not self.kv.allocate_slots(req, 2):  # in-flight token + the new one
                return None
            s = req.num_computed_tokens + 1
            dec.append(ScheduledSeq(req.request_id, [0], s, req.block_ids, True,
                                    sampling_params=req.sampling_params, sample_seq=req.sample_seq + 1,
                                    request=req, swa_block_ids=self._swa(req)))
        if not dec:
            return None
        finished, self._finished_ids = self._finished_ids, []
        if pre:
            return SchedulerOutput("mixed", dec + pre, finished=finished, num_decode=len(dec))
        return SchedulerOutput("decode", dec, finished=finished)

    def _swa(self, req: Request) -> list[int] | None:
        return req.swa_block_ids if self.kv.swa_pool is not None else None

    def _remote_prefill_tokens(self, req: Request) -> int:
        """Prompt positions whose KV comes from the remote engine: all but the last prompt
        token when the transfer covers the whole prompt (prefill -> decode), the transferred
        prefix when it is a shorter conversation prefix (decode -> prefill, the next turn's
        prompt extends it).  A transfer whose token hash does not match this prompt's prefix,
        or shorter than ``remote_pull_threshold`` tokens, is ignored (computed locally)."""
        p = req.kv_transfer_params or {}
        if self.connector is not None and getattr(self.connector, "prefill_all", False):
            return max(0, req.num_prompt_tokens - 1)  # decode benchmarking: every prompt counts as prefilled
        if self.connector is None or not self.connector.is_consumer or not p.get("do_remote_prefill"):
            return 0
        n = min(int(p.get("num_tokens", 0)), req.num_prompt_tokens)
        if "token_hash" in p and token_hash(req.prompt_token_ids[:n]) != p["token_hash"]:
            logger.warning("request %s: transferred KV is for other tokens; computing the prompt here",
                           req.request_id)
            return 0
        threshold = int((getattr(self.connector, "extra", None) or {}).get("remote_pull_threshold", 0))
        if n < max(threshold, 1):
            return 0
        return max(0, min(n, req.num_prompt_tokens - 1))

    def _budget_left(self, pre: list[Request]) -> int:
        return self.max_num_batched_tokens - sum(self._prefill_chunk(r) for r in pre)

    def _prefill_chunk(self, req: Request) -> int:
        remaining = req.num_tokens - req.num_computed_tokens
        if self.chunked:
            return min(remaining, self.max_num_batched_tokens)
        if remaining > self.max_num_batched_tokens:
            raise ValueError("prompt exceeds max_num_batched_tokens and chunked prefill is disabled")
        return remaining

    def _preempt(self, req: Request) -> None:
        self.running.remove(req)
        self.kv.free(req)
        req.num_computed_tokens = 0
        req.spec_token_ids = []
        req.status = RequestStatus.PREEMPTED
        for cb in self.on_preempt:
            cb(req.request_id)
        self.waiting.appendleft(req)
        logger.warning("preempted request %s (KV cache full)", req.request_id)

    # ----------------------------------------------------------------- update
    def update_from_output(self, out: SchedulerOutput, sampled: dict[str, list[int]],
                           now: float | None = None) -> list[Request]:
        """Advance request state after a step.  ``sampled[req_id]`` holds the accepted
        tokens (1 without speculation; 1..k+1 with).  Returns requests that finished."""
        now = now or time.monotonic()
        done = []
        for s in out.seqs:
            req = self.requests.get(s.req_id)
            if req is None:
                continue
            if out.kind in ("prefill", "mixed"):
                req.num_computed_tokens += len(s.token_ids)
            if not s.sample:
                self.kv.cache_full_blocks(req)
                continue
            toks = sampled.get(s.req_id, [])
            if out.kind == "decode":
                # tokens computed = the input token + accepted drafts
                req.num_computed_tokens += max(1, len(toks)) if s.spec_token_ids else 1
            req.spec_token_ids = []
            for t in toks:
                req.output_token_ids.append(int(t))
                req.sample_seq += 1
                if req.metrics.first_token_time is None:
                    req.metrics.first_token_time = now
                req.metrics.token_times.append(now)
                if req.check_stop(self.max_model_len):
                    break
                if req.grammar is not None:  # structured output: advance the grammar
                    if not req.grammar.accept_token(int(t)) or req.grammar.is_terminated():
                        req.status = RequestStatus.FINISHED_STOPPED
                        break
                if req.stop_checker is not None and req.stop_checker(req):  # a stop string appeared
                    req.status = RequestStatus.FINISHED_STOPPED
                    break
            self.kv.cache_full_blocks(req)
            if req.status.finished:
                done.append(req)
                self._finish(req)
        return done
