"""Multi-process executor for tests and tools (``utils/executor.py:428`` ``MPExecutor`` of the
Trainium plugin, re-designed for this framework).

``MPExecutor(world_size=2, tp=2)`` starts one process per rank, initialises
``torch.distributed`` (gloo on CPU, NCCL on GPUs) through a private file rendezvous and
builds the parallel state.  Workers persist across calls and execute tasks from their own
queue:

* ``run(fn, *args)``      call ``fn(ctx, *args)`` on every rank, return the per-rank results;
* ``load(factory, *args)`` build a per-rank object (kept in ``ctx.obj``) for later ``run`` calls;
* ``reinit(tp=, dp=, ...)`` rebuild the parallel state with another layout (same world);
* ``shutdown()``          stop the pool.

Failure detection: a task that raises on any rank makes ``run`` raise ``RankError`` with
the rank and its traceback; a rank process that dies or does not answer within
``timeout_s`` (start-up: ``init_timeout_s``) makes ``run`` raise ``RankError`` as well, after which the pool is torn
down (a fresh executor respawns it).  The ``ctx`` passed to tasks carries ``rank``,
``world_size``, ``ps`` (the parallel state), ``device`` and ``obj``.
"""

from __future__ import annotations

import os
import queue
import time
import traceback
from dataclasses import dataclass, field
from typing import Any, Callable

import torch.multiprocessing as mp


class RankError(RuntimeError):
    def __init__(self, rank: int, msg: str):
        super().__init__(f"rank {rank}: {msg}")
        self.rank = rank


@dataclass
class RankContext:
    rank: int
    world_size: int
    ps: Any = None
    device: Any = None
    obj: Any = None
    store: dict = field(default_factory=dict)


def _worker(rank: int, world_size: int, init_method: str, backend: str, layout: dict, tasks, results,
            timeout_s: float) -> None:
    import torch
    import torch.distributed as dist

    from ..parallel import state as pstate

    ctx = RankContext(rank, world_size)
    try:
        if backend == "nccl":
            torch.cuda.set_device(rank)
            ctx.device = torch.device("cuda", rank)
        else:
            ctx.device = torch.device("cpu")
        pstate.init_distributed_environment(world_size, rank, backend=backend, init_method=init_method,
                                            local_rank=rank, timeout_s=timeout_s)
        ctx.ps = pstate.initialize_parallel_state(backend=backend, timeout_s=timeout_s, **layout)
        results.put((rank, "ready", None))
    except Exception:  # noqa: BLE001
        results.put((rank, "error", traceback.format_exc()))
        return
    while True:
        kind, payload = tasks.get()
        if kind == "stop":
            break
        try:
            if kind == "run":
                fn, args, kwargs = payload
                out = fn(ctx, *args, **kwargs)
            elif kind == "load":
                factory, args, kwargs = payload
                ctx.obj = factory(ctx, *args, **kwargs)
                out = None
            elif kind == "reinit":
                pstate.destroy_parallel_state()
                ctx.ps = pstate.initialize_parallel_state(backend=backend, timeout_s=timeout_s, **payload)
                out = None
            else:
                raise ValueError(f"unknown task {kind}")
            results.put((rank, "ok", out))
        except Exception:  # noqa: BLE001
            results.put((rank, "error", traceback.format_exc()))
    pstate.destroy_parallel_state()
    if dist.is_initialized():
        dist.destroy_process_group()


class MPExecutor:
    def __init__(self, world_size: int, tp: int | None = None, dp: int = 1, backend: str | None = None,
                 timeout_s: float = 120.0, init_timeout_s: float = 300.0, **layout):
        from .rendezvous import FileRendezvous

        self.world_size = world_size
        self.timeout_s = timeout_s
        self.backend = backend or ("nccl" if os.environ.get("VLLM_B200_EXECUTOR_GPU") == "1" else "gloo")
        lay = dict(tp=tp or world_size // dp, dp=dp)
        lay.update(layout)
        self._rdzv = FileRendezvous()
        ctx = mp.get_context("spawn")
        self._results = ctx.Queue()
        self._tasks = [ctx.Queue() for _ in range(world_size)]
        self._procs = [ctx.Process(target=_worker, args=(r, world_size, self._rdzv.init_method, self.backend, lay,
                                                         self._tasks[r], self._results, timeout_s), daemon=True)
                       for r in range(world_size)]
        for p in self._procs:
            p.start()
        self._collect("ready", init_timeout_s)

    # ------------------------------------------------------------------ internals
    def _collect(self, expect: str, timeout_s: float | None = None) -> list:
        timeout_s = self.timeout_s if timeout_s is None else timeout_s
        out: list = [None] * self.world_size
        seen: set[int] = set()
        deadline = time.monotonic() + timeout_s
        errors = []
        while len(seen) < self.world_size:
            left = deadline - time.monotonic()
            if left <= 0:
                missing = [r for r in range(self.world_size) if r not in seen]
                self._kill()
                raise RankError(missing[0] if missing else -1, f"no answer within {timeout_s:.0f}s")
            try:
                rank, status, payload = self._results.get(timeout=min(0.5, left))
            except queue.Empty:
                dead = [(r, p.exitcode) for r, p in enumerate(self._procs) if not p.is_alive() and r not in seen]
                if dead:
                    self._kill()
                    raise RankError(dead[0][0], f"process exited (code {dead[0][1]})")
                continue
            seen.add(rank)
            if status == "error":
                errors.append((rank, payload))
            out[rank] = payload
        if errors:
            rank, tb = errors[0]
            raise RankError(rank, tb)
        return out

    def _send(self, kind: str, payload) -> None:
        if not self._procs:
            raise RuntimeError("executor is shut down")
        for q in self._tasks:
            q.put((kind, payload))

    def _kill(self) -> None:
        for p in self._procs:
            if p.is_alive():
                p.kill()
        for p in self._procs:
            p.join(timeout=5)
        self._procs = []
        self._rdzv.close()

    # -------------------------------------------------------------------- API
    def run(self, fn: Callable, *args, **kwargs) -> list:
        self._send("run", (fn, args, kwargs))
        return self._collect("ok")

    def load(self, factory: Callable, *args, **kwargs) -> None:
        self._send("load", (factory, args, kwargs))
        self._collect("ok")

    def reinit(self, **layout) -> None:
        self._send("reinit", layout)
        self._collect("ok")

    def shutdown(self) -> None:
        if not self._procs:
            return
        self._send("stop", None)
        for p in self._procs:
            p.join(timeout=10)
        self._kill()

    def __enter__(self) -> "MPExecutor":
        return self

    def __exit__(self, *exc) -> None:
        self.shutdown()
