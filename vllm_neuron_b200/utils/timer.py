"""Wall-clock and CUDA-event timers."""

from __future__ import annotations

import time


class Timer:
    """``with Timer() as t: ...; t.elapsed`` (seconds, wall clock)."""

    def __enter__(self) -> "Timer":
        self.t0 = time.perf_counter()
        self.elapsed = 0.0
        return self

    def __exit__(self, *exc) -> None:
        self.elapsed = time.perf_counter() - self.t0


class CudaTimer:
    """Device time of the work issued inside the block on the current stream (ms)."""

    def __enter__(self) -> "CudaTimer":
        import torch

        self.s, self.e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        self.s.record()
        return self

    def __exit__(self, *exc) -> None:
        import torch

        self.e.record()
        torch.cuda.synchronize()
        self.ms = self.s.elapsed_time(self.e)
