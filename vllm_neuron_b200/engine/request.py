"""Request state tracked by the scheduler."""

from __future__ import annotations

import enum
import time
from dataclasses import dataclass, field

from .sampling_params import RequestMetrics, SamplingParams


class RequestStatus(enum.Enum):
    WAITING = 0
    RUNNING = 1
    PREEMPTED = 2
    FINISHED_STOPPED = 3
    FINISHED_LENGTH = 4
    FINISHED_ABORTED = 5
    WAITING_FOR_REMOTE_KVS = 6

    @property
    def finished(self) -> bool:
        return self.value >= 3 and self != RequestStatus.WAITING_FOR_REMOTE_KVS


@dataclass
class Request:
    request_id: str
    prompt_token_ids: list[int]
    sampling_params: SamplingParams
    eos_token_id: int | list[int] | None = None
    prompt: str | None = None
    arrival_time: float = field(default_factory=time.monotonic)
    mm_inputs: list | None = None  # multimodal items (vision)
    kv_transfer_params: dict | None = None
    status: RequestStatus = RequestStatus.WAITING
    output_token_ids: list[int] = field(default_factory=list)
    block_ids: list[int] = field(default_factory=list)
    # sliding-window KV group: logical block table of the windowed layers; entries that fell
    # behind the window are returned to their pool and replaced by the null block 0
    swa_block_ids: list[int] = field(default_factory=list)
    swa_freed: int = 0  # leading entries of swa_block_ids already returned
    num_computed_tokens: int = 0
    num_cached_tokens: int = 0  # prefix-cache hit length at first schedule
    spec_token_ids: list[int] = field(default_factory=list)
    metrics: RequestMetrics = field(default_factory=RequestMetrics)
    stop_reason: int | str | None = None
    sample_seq: int = 0  # deterministic per-request RNG counter
    mm_items: list | None = None  # [{"pixels", "grid", "offset", "n"}] image placeholders in the prompt
    mrope_positions: object = None  # [3, prompt_len] multimodal positions (Qwen3-VL)
    mrope_delta: int = 0  # decode rope position = cache position + delta
    kv_transfer_params_out: dict | None = None  # set by a KV-producer engine when the request finishes
    num_inflight: int = 0  # decode steps launched whose token is not yet known (async scheduling)
    num_inflight_prefill: int = 0  # prompt tokens of a launched, not yet committed step (async mixed steps)
    grammar: object = None  # structured-output matcher (xgrammar), fed every sampled token
    logprobs: list = field(default_factory=list)  # per output token {token id: logprob} (SamplingParams.logprobs)
    stop_checker: object = None  # stop strings: callable(request) -> True when one appeared
    stop_text: str | None = None  # output text cut at the stop string that ended the request

    def __post_init__(self) -> None:
        self.metrics.arrival_time = self.arrival_time

    @property
    def all_token_ids(self) -> list[int]:
        return self.prompt_token_ids + self.output_token_ids

    def token_at(self, i: int) -> int:
        n = len(self.prompt_token_ids)
        return self.prompt_token_ids[i] if i < n else self.output_token_ids[i - n]

    @property
    def num_tokens(self) -> int:
        return len(self.prompt_token_ids) + len(self.output_token_ids)

    @property
    def num_prompt_tokens(self) -> int:
        return len(self.prompt_token_ids)

    @property
    def is_prefill(self) -> bool:
        return self.num_computed_tokens < self.num_tokens - 1 or not self.output_token_ids and \
            self.num_computed_tokens < self.num_prompt_tokens

    @property
    def max_tokens(self) -> int:
        return self.sampling_params.max_tokens or 1 << 30

    def check_stop(self, max_model_len: int) -> bool:
        """Update status from the last sampled token; True when the request finished."""
        sp = self.sampling_params
        n_out = len(self.output_token_ids)
        if n_out == 0:
            return False
        last = self.output_token_ids[-1]
        if n_out >= sp.min_tokens:
            eos = self.eos_token_id
            eos_set = set(eos) if isinstance(eos, (list, tuple)) else ({eos} if eos is not None else set())
            if not sp.ignore_eos and last in eos_set:
                self.status = RequestStatus.FINISHED_STOPPED
                return True
            if sp.stop_token_ids and last in sp.stop_token_ids:
                self.status = RequestStatus.FINISHED_STOPPED
                self.stop_reason = last
                return True
        if n_out >= self.max_tokens or self.num_tokens >= max_model_len:
            self.status = RequestStatus.FINISHED_LENGTH
            return True
        return False
