"""Asynchronous engine front-end for online serving.

A background thread owns the :class:`LLMEngine` and loops ``step()`` while requests are
in flight; API handlers submit requests through a thread-safe queue and receive
per-request outputs on asyncio queues.  This is the role vLLM's AsyncLLM / EngineCore
play for the Trainium plugin (its engine-core loop), collapsed into one process since the
scheduler is deterministic and SPMD across ranks.
"""

from __future__ import annotations

import asyncio
import queue
import threading
import uuid
from typing import AsyncIterator

from ..logging_config import init_logger
from .llm import LLM
from .sampling_params import RequestOutput, SamplingParams

logger = init_logger(__name__)


class AsyncLLM:
    def __init__(self, **engine_kwargs):
        self.llm = LLM(**engine_kwargs)
        self.engine = self.llm.engine
        self._in: queue.Queue = queue.Queue()
        self._streams: dict[str, tuple[asyncio.AbstractEventLoop, asyncio.Queue]] = {}
        self._lock = threading.Lock()
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._loop, name="b200-engine", daemon=True)
        self._thread.start()
        self.profiling = False

    def _loop(self) -> None:
        while not self._stop.is_set():
            try:
                while True:
                    kind, payload = self._in.get_nowait()
                    if kind == "add":
                        rid, ids, sp, mm, kvp = payload
                        try:
                            self.engine.add_request(rid, ids, sp, mm_inputs=mm, kv_transfer_params=kvp)
                        except Exception as e:  # noqa: BLE001  (this request only: the engine keeps serving)
                            logger.error("request %s refused: %s", rid, e)
                            self._fail(rid, e)
                    elif kind == "abort":
                        self.engine.abort_request(payload)
                    elif kind == "call":
                        fn, box, done = payload
                        try:
                            box.append(fn(self.engine))
                        except Exception as e:  # noqa: BLE001
                            box.append(e)
                        done.set()
            except queue.Empty:
                pass
            if not self.engine.has_unfinished_requests():
                try:
                    kind, payload = self._in.get(timeout=0.05)
                    self._in.put((kind, payload))
                except queue.Empty:
                    pass
                continue
            try:
                outs = self.engine.step()
            except Exception as e:  # noqa: BLE001
                logger.exception("engine step failed")
                with self._lock:
                    for rid, (loop, q) in list(self._streams.items()):
                        loop.call_soon_threadsafe(q.put_nowait, e)
                    self._streams.clear()
                continue
            for o in outs:
                with self._lock:
                    ent = self._streams.get(o.request_id)
                if ent is not None:
                    loop, q = ent
                    loop.call_soon_threadsafe(q.put_nowait, o)
                    if o.finished:
                        with self._lock:
                            self._streams.pop(o.request_id, None)

    def _fail(self, rid: str, e: Exception) -> None:
        with self._lock:
            ent = self._streams.pop(rid, None)
        if ent is not None:
            loop, q = ent
            loop.call_soon_threadsafe(q.put_nowait, e if isinstance(e, ValueError) else RuntimeError(str(e)))

    async def generate(self, prompt_token_ids: list[int], sampling_params: SamplingParams,
                       request_id: str | None = None, mm_inputs: list | None = None,
                       kv_transfer_params: dict | None = None) -> AsyncIterator[RequestOutput]:
        rid = request_id or uuid.uuid4().hex
        loop = asyncio.get_running_loop()
        q: asyncio.Queue = asyncio.Queue()
        with self._lock:
            self._streams[rid] = (loop, q)
        self._in.put(("add", (rid, list(prompt_token_ids), sampling_params, mm_inputs, kv_transfer_params)))
        try:
            while True:
                item = await q.get()
                if isinstance(item, Exception):
                    raise item
                yield item
                if item.finished:
                    return
        except asyncio.CancelledError:
            self._in.put(("abort", rid))
            raise

    def call(self, fn, timeout: float = 60.0):
        """Run ``fn(engine)`` on the engine thread between steps and return its result."""
        box: list = []
        done = threading.Event()
        self._in.put(("call", (fn, box, done)))
        if not done.wait(timeout):
            raise RuntimeError("engine did not answer")
        if isinstance(box[0], Exception):
            raise box[0]
        return box[0]

    def abort(self, request_id: str) -> None:
        self._in.put(("abort", request_id))

    def shutdown(self) -> None:
        self._stop.set()
        self._thread.join(timeout=10)
        self.llm.shutdown()
