"""Profiling of serving steps (``vllm/worker/neuron_profiler.py`` of the Trainium plugin).

``additional_config = {"neuron_profiler": {...}}`` (the reference's key) or ``{"profiler": {...}}``:

* ``activities``: any of "cpu", "cuda" (default both; the reference's "device_profile" and
  "system_profile" map to "cuda" and "cpu");
* ``output_dir``: where traces are written (default ``<tmpdir>/vllm_b200_profiles``, outside
  any source tree);
* ``record_shapes``, ``with_stack``: passed to ``torch.profiler``;
* ``max_steps``: stop automatically after this many engine steps (0 = until stopped).

``/start_profile`` and ``/stop_profile`` on the server, or ``LLM.start_profile()`` /
``LLM.stop_profile()``, bracket the steps to record; ``stop`` writes a Chrome trace
(``trace_<rank>_<time>.json``) and a per-kernel summary table (``summary_<rank>_<time>.txt``,
device time per kernel, the place to look first).  Timings taken under the profiler are for
attribution, not for reporting throughput.
"""

from __future__ import annotations

import os
import tempfile
import time
from dataclasses import dataclass, field

_ALIASES = {"device_profile": "cuda", "system_profile": "cpu"}


@dataclass
class ProfilerConfig:
    activities: list = field(default_factory=lambda: ["cpu", "cuda"])
    output_dir: str = field(default_factory=lambda: os.path.join(tempfile.gettempdir(), "vllm_b200_profiles"))
    record_shapes: bool = False
    with_stack: bool = False
    max_steps: int = 0

    @classmethod
    def from_dict(cls, d: dict | None) -> "ProfilerConfig":
        d = dict(d or {})
        acts = [_ALIASES.get(a, a) for a in d.pop("activities", ["cpu", "cuda"])]
        bad = [a for a in acts if a not in ("cpu", "cuda")]
        if bad:
            raise ValueError(f"profiler activities must be 'cpu' / 'cuda', got {bad}")
        d.pop("neuron_cores", None)  # reference-only keys
        d.pop("sys_trace_max_events_per_nc", None)
        known = set(cls.__dataclass_fields__)
        unknown = set(d) - known
        if unknown:
            raise ValueError(f"unknown profiler keys {sorted(unknown)}")
        return cls(activities=sorted(set(acts)), **d)


class Profiler:
    def __init__(self, cfg: ProfilerConfig | None = None, rank: int = 0):
        self.cfg = cfg or ProfilerConfig()
        self.rank = rank
        self._prof = None
        self.steps = 0

    @property
    def active(self) -> bool:
        return self._prof is not None

    def start(self) -> None:
        import torch

        if self._prof is not None:
            raise RuntimeError("profiler already running")
        acts = []
        if "cpu" in self.cfg.activities:
            acts.append(torch.profiler.ProfilerActivity.CPU)
        if "cuda" in self.cfg.activities and torch.cuda.is_available():
            acts.append(torch.profiler.ProfilerActivity.CUDA)
        self._prof = torch.profiler.profile(activities=acts, record_shapes=self.cfg.record_shapes,
                                            with_stack=self.cfg.with_stack)
        self._prof.__enter__()
        self.steps = 0

    def step(self) -> None:
        """Called once per engine step while active (auto-stop after ``max_steps``)."""
        if self._prof is None:
            return
        self.steps += 1
        if self.cfg.max_steps and self.steps >= self.cfg.max_steps:
            self.stop()

    def stop(self) -> dict:
        if self._prof is None:
            raise RuntimeError("profiler not running")
        prof, self._prof = self._prof, None
        prof.__exit__(None, None, None)
        os.makedirs(self.cfg.output_dir, exist_ok=True)
        stamp = int(time.time() * 1000)
        trace = os.path.join(self.cfg.output_dir, f"trace_{self.rank}_{stamp}.json")
        prof.export_chrome_trace(trace)
        summary = os.path.join(self.cfg.output_dir, f"summary_{self.rank}_{stamp}.txt")
        try:
            key = "self_cuda_time_total" if "cuda" in self.cfg.activities else "self_cpu_time_total"
            table = prof.key_averages().table(sort_by=key, row_limit=40)
        except Exception:  # noqa: BLE001  (no device events recorded)
            table = prof.key_averages().table(sort_by="self_cpu_time_total", row_limit=40)
        with open(summary, "w") as f:
            f.write(table)
        return {"trace": trace, "summary": summary, "steps": self.steps}
