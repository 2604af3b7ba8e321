"""Safetensors checkpoint reading.

Streams ``(name, tensor)`` pairs from every ``*.safetensors`` file of a model
directory (``SafetensorsCheckpoint``, ``vllm_neuron/utils/checkpoints.py:143``).
Files are memory-mapped; a background thread reads the next file ahead while the
caller transforms and copies the current one to the GPU, the same disk -> page
cache -> transform -> device pipelining as ``load_sharded_pipelined`` (``:273``).
"""

from __future__ import annotations

import glob
import json
import os
import queue
import threading
from typing import Iterator

import torch


def list_checkpoint_files(path: str) -> list[str]:
    idx = os.path.join(path, "model.safetensors.index.json")
    if os.path.exists(idx):
        with open(idx) as f:
            files = sorted(set(json.load(f)["weight_map"].values()))
        return [os.path.join(path, x) for x in files]
    return sorted(glob.glob(os.path.join(path, "*.safetensors")))


def _prefetch(fn: str) -> None:
    try:
        with open(fn, "rb") as f:
            while f.read(64 << 20):
                pass
    except OSError:
        pass


class SafetensorsCheckpoint:
    def __init__(self, path: str, prefetch: bool = True):
        self.path = path
        self.files = list_checkpoint_files(path)
        if not self.files:
            raise FileNotFoundError(f"no safetensors files under {path}")
        self.prefetch = prefetch

    def keys(self) -> list[str]:
        from safetensors import safe_open

        out = []
        for fn in self.files:
            with safe_open(fn, framework="pt") as f:
                out.extend(f.keys())
        return out

    def __iter__(self) -> Iterator[tuple[str, torch.Tensor]]:
        from safetensors import safe_open

        q: queue.Queue = queue.Queue()
        if self.prefetch and len(self.files) > 1:
            def run():
                for fn in self.files[1:]:
                    _prefetch(fn)
                    q.put(fn)

            threading.Thread(target=run, daemon=True).start()
        for fn in self.files:
            with safe_open(fn, framework="pt") as f:
                for k in f.keys():
                    yield k, f.get_tensor(k)


def save_state_dict(sd: dict[str, torch.Tensor], path: str, config: dict | None = None,
                    max_shard_bytes: int = 4 << 30) -> None:
    """Write a (possibly sharded) safetensors checkpoint plus config.json."""
    from safetensors.torch import save_file

    os.makedirs(path, exist_ok=True)
    shards, cur, size = [], {}, 0
    for k, v in sd.items():
        nb = v.numel() * v.element_size()
        if cur and size + nb > max_shard_bytes:
            shards.append(cur)
            cur, size = {}, 0
        cur[k] = v.contiguous()
        size += nb
    if cur:
        shards.append(cur)
    wm = {}
    for i, sh in enumerate(shards):
        fn = f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors" if len(shards) > 1 else "model.safetensors"
        save_file(sh, os.path.join(path, fn))
        for k in sh:
            wm[k] = fn
    if len(shards) > 1:
        with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
            json.dump({"metadata": {}, "weight_map": wm}, f)
    if config is not None:
        with open(os.path.join(path, "config.json"), "w") as f:
            json.dump(config, f, indent=1)
