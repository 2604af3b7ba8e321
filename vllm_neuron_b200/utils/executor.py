"""Multi-process executor for tests and tools (``utils/executor.py:428`` ``MPExecutor`` of the
Trainium plugin, re-designed for this framework).

``MPExecutor(world_size=2, tp=2)`` starts one process per rank, initialises
``torch.distributed`` (gloo on CPU, NCCL on GPUs) through a private file rendezvous and
builds the parallel state.  Workers persist across calls and execute tasks from their own
queue:

* ``run(fn, *args)``      call ``fn(ctx, *args)`` on every rank, return the per-rank results;
* ``load(factory, *args)`` build a per-rank object (kept in ``ctx.obj``) for later ``run`` calls;
* ``run_per_rank(fn, [args_0, args_1, ...])`` call ``fn(ctx, *args_r)`` with each rank's own
  arguments (e.g. the shard of an input that rank r owns);
* ``reinit(tp=, dp=, ...)`` rebuild the parallel state with another layout (same world);
* ``start_profile(dir)`` / ``stop_profile()`` record every rank with ``torch.profiler`` (CPU, and
  CUDA activity on GPU ranks) and write one Chrome trace per rank
  (reference: ``utils/executor.py:618-732``);
* ``shutdown()``          stop the pool.

``MPExecutor.shared(world_size, **layout)`` returns a pooled executor that later calls with the
same world size reuse (re-laid-out with ``reinit`` when the layout differs), so a test suite
pays for process start-up and rendezvous once per world size (``_WorkerPool``, reference
``utils/executor.py:100``).  ``nnodes`` simulates a multi-node job on one host: ranks are dealt
to nodes in contiguous blocks and ``ctx.node_rank`` / ``ctx.local_rank`` / ``ctx.nnodes`` tell a
task where its rank sits.

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
    nnodes: int = 1
    node_rank: int = 0
    local_rank: int = 0
    profiler: Any = None


def _start_profile(ctx: RankContext, out_dir: str) -> None:
    import torch

    acts = [torch.profiler.ProfilerActivity.CPU]
    if ctx.device is not None and ctx.device.type == "cuda":
        acts.append(torch.profiler.ProfilerActivity.CUDA)
    ctx.store["profile_dir"] = out_dir
    ctx.profiler = torch.profiler.profile(activities=acts, record_shapes=True)
    ctx.profiler.__enter__()


def _stop_profile(ctx: RankContext) -> str | None:
    if ctx.profiler is None:
        return None
    ctx.profiler.__exit__(None, None, None)
    out_dir = ctx.store.pop("profile_dir")
    os.makedirs(out_dir, exist_ok=True)
    path = os.path.join(out_dir, f"trace_rank{ctx.rank}.json")
    ctx.profiler.export_chrome_trace(path)
    ctx.profiler = None
    return path


def _worker(rank: int, world_size: int, init_method: str, backend: str, layout: dict, tasks, results,
            timeout_s: float, nnodes: int = 1) -> None:
    import torch
    import torch.distributed as dist

    from ..parallel import state as pstate

    per_node = world_size // nnodes
    ctx = RankContext(rank, world_size, nnodes=nnodes, node_rank=rank // per_node, local_rank=rank % per_node)
    try:
        if backend == "nccl":
            torch.cuda.set_device(rank)
            ctx.device = torch.device("cuda", rank)
        else:
            ctx.device = torch.device("cpu")
        pstate.init_distributed_environment(world_size, rank, backend=backend, init_method=init_method,
                                            local_rank=rank, timeout_s=timeout_s)
        ctx.ps = pstate.initialize_parallel_state(backend=backend, timeout_s=timeout_s, nnodes=nnodes, **layout)
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
            elif kind == "run_per_rank":
                fn, per_rank, kwargs = payload
                out = fn(ctx, *per_rank[rank], **kwargs)
            elif kind == "start_profile":
                _start_profile(ctx, payload)
                out = None
            elif kind == "stop_profile":
                out = _stop_profile(ctx)
            elif kind == "load":
                factory, args, kwargs = payload
                ctx.obj = factory(ctx, *args, **kwargs)
                out = None
            elif kind == "reinit":
                pstate.destroy_parallel_state()
                ctx.ps = pstate.initialize_parallel_state(backend=backend, timeout_s=timeout_s, nnodes=nnodes,
                                                          **payload)
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
    _pool: dict = {}

    def __init__(self, world_size: int, tp: int | None = None, dp: int = 1, backend: str | None = None,
                 timeout_s: float = 120.0, init_timeout_s: float = 300.0, nnodes: int = 1, **layout):
        from .rendezvous import FileRendezvous

        if nnodes < 1 or world_size % nnodes:
            raise ValueError(f"world_size {world_size} is not a multiple of nnodes {nnodes}")
        self.world_size = world_size
        self.nnodes = nnodes
        self.timeout_s = timeout_s
        self.backend = backend or ("nccl" if os.environ.get("VLLM_B200_EXECUTOR_GPU") == "1" else "gloo")
        lay = dict(tp=tp or world_size // dp, dp=dp)
        lay.update(layout)
        self.layout = lay
        self._rdzv = FileRendezvous()
        ctx = mp.get_context("spawn")
        self._results = ctx.Queue()
        self._tasks = [ctx.Queue() for _ in range(world_size)]
        self._procs = [ctx.Process(target=_worker, args=(r, world_size, self._rdzv.init_method, self.backend, lay,
                                                         self._tasks[r], self._results, timeout_s, nnodes),
                                  daemon=True)
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

    def run_per_rank(self, fn: Callable, per_rank_args: list, **kwargs) -> list:
        if len(per_rank_args) != self.world_size:
            raise ValueError(f"{len(per_rank_args)} argument sets for {self.world_size} ranks")
        per_rank = [tuple(a) if isinstance(a, (tuple, list)) else (a,) for a in per_rank_args]
        self._send("run_per_rank", (fn, per_rank, kwargs))
        return self._collect("ok")

    def reinit(self, **layout) -> None:
        self._send("reinit", layout)
        self._collect("ok")
        self.layout = dict(layout)

    def start_profile(self, out_dir: str) -> None:
        self._send("start_profile", out_dir)
        self._collect("ok")

    def stop_profile(self) -> list:
        """Per-rank Chrome trace paths."""
        self._send("stop_profile", None)
        return self._collect("ok")

    @classmethod
    def shared(cls, world_size: int, tp: int | None = None, dp: int = 1, **layout) -> "MPExecutor":
        """A pooled executor per (world size, backend); reused and re-laid-out across calls.
        ``shutdown_shared()`` (also run at interpreter exit) stops them."""
        lay = dict(tp=tp or world_size // dp, dp=dp)
        lay.update(layout)
        backend = "nccl" if os.environ.get("VLLM_B200_EXECUTOR_GPU") == "1" else "gloo"
        ex = cls._pool.get((world_size, backend))
        if ex is not None and not ex._procs:
            ex = None
        if ex is None:
            if not cls._pool:
                import atexit

                atexit.register(cls.shutdown_shared)
            ex = cls(world_size, backend=backend, **lay)
            cls._pool[(world_size, backend)] = ex
        elif ex.layout != lay:
            ex.reinit(**lay)
        return ex

    @classmethod
    def shutdown_shared(cls) -> None:
        for ex in list(cls._pool.values()):
            ex.shutdown()
        cls._pool.clear()

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
