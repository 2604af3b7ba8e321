"""``LLM``: the offline entry point, with vLLM's constructor arguments and
``generate`` signature for the supported features."""

from __future__ import annotations

import os
from typing import Sequence

import torch.multiprocessing as mp

from ..config import EngineConfig
from ..logging_config import init_logger
from .llm_engine import LLMEngine, _follower_main
from .sampling_params import RequestOutput, SamplingParams

logger = init_logger(__name__)


def stop_workers(procs: list, grace_s: float = 30.0, term_timeout_s: float | None = None) -> list[str]:
    """Stop worker processes that were told to shut down: wait up to ``grace_s`` (in total) for
    them to exit, send SIGTERM to the ones still running, and SIGKILL whatever is left after
    ``term_timeout_s`` (default ``VLLM_B200_WORKER_TERMINATION_TIMEOUT``), so a wedged worker
    cannot hold the shutdown (the reference patches the same SIGTERM -> SIGKILL escalation,
    ``vllm/platform.py:783``).  Returns how each process ended ("exited", "terminated",
    "killed")."""
    import time

    from .. import envs

    if term_timeout_s is None:
        term_timeout_s = float(envs.VLLM_B200_WORKER_TERMINATION_TIMEOUT)
    deadline = time.monotonic() + grace_s
    how = ["exited"] * len(procs)
    for p in procs:
        p.join(timeout=max(0.0, deadline - time.monotonic()))
    for i, p in enumerate(procs):
        if p.is_alive():
            p.terminate()
            how[i] = "terminated"
    deadline = time.monotonic() + term_timeout_s
    for i, p in enumerate(procs):
        if how[i] == "terminated":
            p.join(timeout=max(0.0, deadline - time.monotonic()))
            if p.is_alive():
                p.kill()
                p.join(timeout=5)
                how[i] = "killed"
    return how


def merge_samples(request_id: str, outs: list[RequestOutput]) -> RequestOutput:
    """One RequestOutput with the n completions of a prompt (index = sample number)."""
    if len(outs) == 1:
        return outs[0]
    first = outs[0]
    comps = []
    for j, o in enumerate(outs):
        c = o.outputs[0]
        c.index = j
        comps.append(c)
    return RequestOutput(request_id, first.prompt, first.prompt_token_ids, comps, all(o.finished for o in outs),
                         first.metrics, first.num_cached_tokens, first.kv_transfer_params)


class LLM:
    """Example::

        llm = LLM(model="/path/to/gpt-oss-120b", tensor_parallel_size=8, max_model_len=8192,
                  additional_config={"neuron_config": {"quantization": "mxfp4"}})
        outs = llm.generate(prompt_token_ids=[[1, 2, 3]], sampling_params=SamplingParams(max_tokens=32))

    ``model`` may also be omitted when ``hf_config`` (a config.json dict) is given;
    ``load_format="dummy"`` initialises random weights.  Under ``torchrun`` (``RANK``
    and ``WORLD_SIZE`` set) every rank constructs an ``LLM`` with ``spmd=True`` and
    submits the same requests; otherwise ``tensor_parallel_size > 1`` spawns the
    follower ranks itself."""

    def __init__(self, model: str | None = None, spmd: bool = False, tokenizer: str | None = None, **kwargs):
        cfg = EngineConfig.create(model=model, **kwargs)
        self.cfg = cfg
        ws = cfg.world_size
        self._procs = []
        self._rdzv = None
        if spmd or (ws > 1 and "RANK" in os.environ and int(os.environ.get("WORLD_SIZE", "1")) == ws):
            rank = int(os.environ.get("RANK", "0"))
            local = int(os.environ.get("LOCAL_RANK", rank))
            self.engine = LLMEngine(cfg, rank, ws, local, mode="spmd" if ws > 1 else "single")
        elif ws > 1:
            from ..utils.rendezvous import FileRendezvous

            # ranks meet through a private file store: no port to race for
            self._rdzv = FileRendezvous()
            self._rdzv.export()
            port = 0
            ctx = mp.get_context("spawn")
            for r in range(1, ws):
                p = ctx.Process(target=_follower_main, args=(cfg, r, ws, port), daemon=True)
                p.start()
                self._procs.append(p)
            self.engine = LLMEngine(cfg, 0, ws, 0, mode="driver")
        else:
            self.engine = LLMEngine(cfg, 0, 1, 0, mode="single")
        self._tok = None
        self._tok_path = tokenizer or model
        self._counter = 0

    # ----------------------------------------------------------------- tokenizer
    def get_tokenizer(self):
        if self._tok is None:
            if not self._tok_path:
                raise ValueError("no tokenizer available: pass prompt_token_ids")
            from transformers import AutoTokenizer

            self._tok = AutoTokenizer.from_pretrained(self._tok_path)
        return self._tok

    # ------------------------------------------------------------------ generate
    def generate(self, prompts: Sequence[str] | str | None = None,
                 sampling_params: SamplingParams | Sequence[SamplingParams] | None = None,
                 prompt_token_ids: Sequence[Sequence[int]] | None = None, use_tqdm: bool = False,
                 multi_modal_data: Sequence[dict] | None = None) -> list[RequestOutput]:
        kvps = None
        if prompt_token_ids is None:
            if prompts is None:
                raise ValueError("either prompts or prompt_token_ids is required")
            if isinstance(prompts, str):
                prompts = [prompts]
            if prompts and isinstance(prompts[0], dict):  # {"prompt_token_ids": [...]} items
                prompt_token_ids = [p["prompt_token_ids"] for p in prompts]
                multi_modal_data = [p.get("multi_modal_data") for p in prompts]
                kvps = [p.get("kv_transfer_params") for p in prompts]
                prompts = None
            else:
                tok = self.get_tokenizer()
                prompt_token_ids = [tok.encode(p) for p in prompts]
        n = len(prompt_token_ids)
        if sampling_params is None:
            sampling_params = SamplingParams()
        sps = list(sampling_params) if isinstance(sampling_params, (list, tuple)) else [sampling_params] * n
        ids = []  # per prompt: the request ids of its n samples
        for i, ptoks in enumerate(prompt_token_ids):
            rid = f"req-{self._counter}"
            self._counter += 1
            mm = multi_modal_data[i] if multi_modal_data else None
            # parallel sampling: n child requests of one prompt (their request-keyed uniforms
            # differ, and with prefix caching they share the prompt's KV blocks)
            children = [rid] if sps[i].n == 1 else [f"{rid}#{j}" for j in range(sps[i].n)]
            for cid in children:
                self.engine.add_request(cid, list(ptoks), sps[i], prompt=prompts[i] if prompts else None,
                                        mm_inputs=[mm] if mm else None,
                                        kv_transfer_params=kvps[i] if kvps else None)
            ids.append(children)
        results: dict[str, RequestOutput] = {}
        while self.engine.has_unfinished_requests():
            for o in self.engine.step():
                if o.finished:
                    results[o.request_id] = o
        outs = [merge_samples(rid[0].split("#")[0], [results[c] for c in rid]) for rid in ids]
        if self._tok is not None or (self._tok_path and os.path.exists(os.path.join(self._tok_path,
                                                                                    "tokenizer.json"))):
            try:
                tok = self.get_tokenizer()
                for o in outs:
                    for c in o.outputs:
                        if not isinstance(c.stop_reason, str):  # a stop string already cut the text
                            c.text = tok.decode(c.token_ids)
            except Exception:  # noqa: BLE001
                pass
        return outs

    def start_profile(self) -> None:
        """Record the following engine steps (see ``vllm_neuron_b200.profiler``)."""
        self.engine.start_profile()

    def stop_profile(self) -> dict:
        return self.engine.stop_profile()

    def shutdown(self) -> None:
        self.engine.shutdown()
        stop_workers(self._procs)
        self._procs = []
        if getattr(self, "_rdzv", None) is not None:
            self._rdzv.close()
            self._rdzv = None

    def __del__(self):  # pragma: no cover
        try:
            if self._procs:
                self.shutdown()
        except Exception:
            pass
