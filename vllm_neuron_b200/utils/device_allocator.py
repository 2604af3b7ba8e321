"""Hands out GPUs to parallel test workers (the reference's ``utils/core_allocator.py``
``CoreAllocator`` ``:36``, which hands out contiguous NeuronCores).

State lives in a JSON file guarded by ``flock``: ``{device index: owner pid}``.  ``acquire(n)``
takes ``n`` contiguous free devices (entries of dead processes are reclaimed first) and waits up
to ``timeout_s`` for them; ``release`` returns them.  Use as a context manager to release on
exit, and export the indices as ``CUDA_VISIBLE_DEVICES`` for the worker."""

from __future__ import annotations

import contextlib
import fcntl
import json
import os
import time


class DeviceAllocator:
    def __init__(self, num_devices: int, state_path: str = "/tmp/vllm_b200_devices.json"):
        if num_devices < 1:
            raise ValueError("num_devices must be >= 1")
        self.n = num_devices
        self.path = state_path
        self.lock_path = state_path + ".lock"
        self.held: list[int] = []

    @contextlib.contextmanager
    def _locked(self):
        with open(self.lock_path, "a+") as lf:
            fcntl.flock(lf, fcntl.LOCK_EX)
            try:
                yield
            finally:
                fcntl.flock(lf, fcntl.LOCK_UN)

    def _read(self) -> dict:
        try:
            with open(self.path) as f:
                return {int(k): int(v) for k, v in json.load(f).items()}
        except (OSError, ValueError):
            return {}

    def _write(self, state: dict) -> None:
        tmp = self.path + f".tmp{os.getpid()}"
        with open(tmp, "w") as f:
            json.dump({str(k): v for k, v in state.items()}, f)
        os.replace(tmp, self.path)

    @staticmethod
    def _alive(pid: int) -> bool:
        try:
            os.kill(pid, 0)
        except ProcessLookupError:
            return False
        except PermissionError:
            return True
        return True

    def acquire(self, count: int = 1, timeout_s: float = 600.0, poll_s: float = 0.5) -> list[int]:
        if count < 1 or count > self.n:
            raise ValueError(f"cannot acquire {count} of {self.n} devices")
        deadline = time.monotonic() + timeout_s
        while True:
            with self._locked():
                state = {d: p for d, p in self._read().items() if self._alive(p)}  # reclaim dead owners
                for start in range(0, self.n - count + 1):
                    run = list(range(start, start + count))
                    if all(d not in state for d in run):
                        for d in run:
                            state[d] = os.getpid()
                        self._write(state)
                        self.held += run
                        return run
                self._write(state)
            if time.monotonic() > deadline:
                raise TimeoutError(f"no {count} contiguous free devices within {timeout_s:.0f}s")
            time.sleep(poll_s)

    def release(self, devices: list[int] | None = None) -> None:
        devices = list(self.held if devices is None else devices)
        with self._locked():
            state = self._read()
            for d in devices:
                if state.get(d) == os.getpid():
                    del state[d]
            self._write(state)
        self.held = [d for d in self.held if d not in devices]

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.release()
