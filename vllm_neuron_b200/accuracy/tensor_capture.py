"""Capture intermediate tensors of a model during serving (``accuracy/tensor_capture.py`` of
the Trainium plugin, ``NeuronConfig.tensor_capture_config``).

Patterns name modules by their qualified names with integer ranges expanded:
``"layers.0-3.mlp"`` -> ``layers.0.mlp`` .. ``layers.3.mlp``; a pattern without a range must
match a module name exactly.  Every forward pass of the model is one step; the output (the
first tensor of a tuple output) of every matched module is copied to host memory, and
``flush(meta)`` writes the step to ``<capture_dir>/step_<n>_rank<r>.pt`` as
``{"meta": {...request ids, positions, prefill flag...}, "tensors": {name: tensor}}``.
CUDA graphs are disabled while capturing (eager steps run the hooks).
``capture_filter`` optionally keeps only steps of the listed kinds ("prefill", "decode").
"""

from __future__ import annotations

import os
import re

import torch
import torch.nn as nn


def expand_patterns(patterns: list[str]) -> list[str]:
    out = []
    for p in patterns:
        m = re.search(r"(\d+)-(\d+)", p)
        if not m:
            out.append(p)
            continue
        lo, hi = int(m.group(1)), int(m.group(2))
        for i in range(lo, hi + 1):
            out += expand_patterns([p[:m.start()] + str(i) + p[m.end():]])
    return out


def _first_tensor(x):
    if isinstance(x, torch.Tensor):
        return x
    if isinstance(x, (tuple, list)):
        for y in x:
            t = _first_tensor(y)
            if t is not None:
                return t
    return None


class TensorCapture:
    def __init__(self, model: nn.Module, patterns: list[str], capture_dir: str, rank: int = 0,
                 capture_filter: list[str] | None = None):
        self.names = expand_patterns(patterns)
        mods = dict(model.named_modules())
        missing = [n for n in self.names if n not in mods]
        if missing:
            raise KeyError(f"tensor capture: no module named {missing[:4]}")
        self.dir = capture_dir
        self.rank = rank
        self.filter = set(capture_filter) if capture_filter else None
        self.step = 0
        self.buf: dict[str, torch.Tensor] = {}
        self.handles = [mods[n].register_forward_hook(self._hook(n)) for n in self.names]
        os.makedirs(capture_dir, exist_ok=True)

    def _hook(self, name):
        def fn(module, inputs, output):
            t = _first_tensor(output)
            if t is not None:
                self.buf[name] = t.detach().to("cpu", copy=True)
        return fn

    def flush(self, meta: dict) -> str | None:
        """Write the tensors captured since the last flush (one model step)."""
        kind = meta.get("kind")
        path = None
        if self.buf and (self.filter is None or kind in self.filter):
            path = os.path.join(self.dir, f"step_{self.step:05d}_rank{self.rank}.pt")
            torch.save({"meta": meta, "tensors": self.buf}, path)
        self.buf = {}
        self.step += 1
        return path

    def remove(self) -> None:
        for h in self.handles:
            h.remove()
        self.handles = []


def load_captures(capture_dir: str, rank: int = 0) -> list[dict]:
    files = sorted(f for f in os.listdir(capture_dir) if f.endswith(f"_rank{rank}.pt"))
    return [torch.load(os.path.join(capture_dir, f), weights_only=False) for f in files]
