"""Sampling parameters and request outputs (the subset of vLLM's API the engine serves)."""

from __future__ import annotations

from dataclasses import dataclass, field


@dataclass
class SamplingParams:
    """Same field names and defaults as ``vllm.SamplingParams`` for the supported knobs."""

    n: int = 1
    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = 0  # 0 or -1: no top-k limit (bounded by max_top_k on device)
    max_tokens: int | None = 16
    min_tokens: int = 0
    seed: int | None = None
    stop_token_ids: list[int] | None = None
    ignore_eos: bool = False
    logprobs: int | None = None
    detokenize: bool = False
    # grammar constraint (``engine/structured_output.py``): a StructuredOutputsParams or a
    # dict with one of json / regex / choice / grammar / json_object
    structured_outputs: object = None
    # stop strings: generation ends when the decoded output contains one (the text is cut
    # before it unless include_stop_str_in_output)
    stop: list[str] | str | None = None
    include_stop_str_in_output: bool = False

    def __post_init__(self) -> None:
        if self.temperature < 0:
            raise ValueError("temperature must be >= 0")
        if not 0 < self.top_p <= 1:
            raise ValueError("top_p must be in (0, 1]")
        if self.top_k < -1:
            raise ValueError("top_k must be -1, 0 or positive")
        if self.max_tokens is not None and self.max_tokens < 1:
            raise ValueError("max_tokens must be >= 1")
        if self.n < 1:
            raise ValueError("n must be >= 1")
        if isinstance(self.stop, str):
            self.stop = [self.stop]
        if self.stop is not None:
            self.stop = [x for x in self.stop if x]
        if self.structured_outputs is not None:
            from .structured_output import StructuredOutputsParams

            self.structured_outputs = StructuredOutputsParams.from_any(self.structured_outputs)

    @property
    def greedy(self) -> bool:
        return self.temperature == 0.0


@dataclass
class CompletionOutput:
    index: int
    text: str
    token_ids: list[int]
    finish_reason: str | None = None
    logprobs: list | None = None
    stop_reason: int | str | None = None  # the stop token id or stop string that ended the request


@dataclass
class RequestMetrics:
    arrival_time: float = 0.0
    first_scheduled_time: float | None = None
    first_token_time: float | None = None
    finished_time: float | None = None
    token_times: list[float] = field(default_factory=list)


@dataclass
class RequestOutput:
    request_id: str
    prompt: str | None
    prompt_token_ids: list[int]
    outputs: list[CompletionOutput]
    finished: bool
    metrics: RequestMetrics | None = None
    num_cached_tokens: int = 0
    kv_transfer_params: dict | None = None
