"""vLLM scheduler with this framework's step policy (``scheduler_config.scheduler_cls``).

The Trainium plugin replaces vLLM's scheduler with one that never mixes prefill and decode
work in a step (``vllm_neuron/vllm/core/scheduler.py:785`` ``NeuronScheduler.schedule``).
This framework's own scheduler (``engine/scheduler.py``) has the same rule for a B200
reason: a decode step of single-token requests replays a captured CUDA graph per batch
bucket, and one prompt chunk in the batch would send the whole step down the varlen path.
So here a step is either

* prefill work (running requests still inside their prompt, then newly admitted ones), with
  the decoding requests left out of the batch for that step, or
* every decoding request (one token each).

vLLM's ``Scheduler.schedule`` does the admission, KV block allocation, prefix-cache lookup
and preemption; this class only decides which running requests it may see.  Prefill wins
while there is admissible prompt work; if such a step schedules nothing (e.g. the first
waiting prompt does not fit in the free KV blocks) the next step sees every request.
"""

from __future__ import annotations

try:
    from vllm.v1.core.sched.async_scheduler import AsyncScheduler
    from vllm.v1.core.sched.scheduler import Scheduler
except Exception:  # noqa: BLE001 - vLLM absent: the classes are then unusable by vLLM
    class Scheduler:  # type: ignore[no-redef]
        pass

    class AsyncScheduler(Scheduler):  # type: ignore[no-redef]
        pass


def _in_prompt(req) -> bool:
    return req.num_computed_tokens < req.num_prompt_tokens


class B200VllmScheduler(Scheduler):
    _mixed_next = False  # the last prefill-only step scheduled nothing: let every request in

    def _prefill_admissible(self) -> bool:
        if not self.waiting or len(self.running) >= self.max_num_running_reqs:
            return False
        req = self.waiting.peek_request() if hasattr(self.waiting, "peek_request") else next(iter(self.waiting))
        bs = self.cache_config.block_size
        need = min(req.num_tokens, self.scheduler_config.max_num_batched_tokens)
        free = self.kv_cache_manager.block_pool.get_num_free_blocks()
        return free >= -(-need // bs)

    def schedule(self):
        prompt = [r for r in self.running if _in_prompt(r)]
        decoding = [r for r in self.running if not _in_prompt(r)]
        prefill_step = bool(prompt) or self._prefill_admissible()
        if self._mixed_next or not prefill_step or not decoding:
            self._mixed_next = False
            return super().schedule()
        # prefill step: vLLM's scheduler sees the prompt requests (and the waiting queue) only
        self.running = prompt
        self.max_num_running_reqs -= len(decoding)
        try:
            out = super().schedule()
        finally:
            self.max_num_running_reqs += len(decoding)
            self.running = self.running + decoding
        if out.total_num_scheduled_tokens == 0:
            self._mixed_next = True
        return out


class B200VllmAsyncScheduler(B200VllmScheduler, AsyncScheduler):
    """The same policy over vLLM's asynchronous scheduler (output placeholders)."""
