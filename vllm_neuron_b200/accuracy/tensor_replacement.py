"""Replace intermediate tensors with reference values (``accuracy/tensor_replacement.py`` of the
Trainium plugin, ``NeuronConfig.tensor_replacement_config``).

Used to localise a divergence: feeding the reference model's activation of one module into
the engine shows whether the error originates before or after that module.  ``tensors`` is
a list with one entry per model step (forward pass); each entry maps module names to the
tensor that replaces that module's output (same shape), e.g. the "tensors" of steps written
by :mod:`tensor_capture` from a reference run.  Steps beyond the list run unmodified.
"""

from __future__ import annotations

import torch
import torch.nn as nn


class TensorReplacer:
    def __init__(self, model: nn.Module, tensors: list[dict]):
        self.steps = tensors
        self.step = 0
        mods = dict(model.named_modules())
        names = sorted({n for s in tensors for n in s})
        missing = [n for n in names if n not in mods]
        if missing:
            raise KeyError(f"tensor replacement: no module named {missing[:4]}")
        self.handles = [mods[n].register_forward_hook(self._hook(n)) for n in names]
        self.replaced = 0

    def _hook(self, name):
        def fn(module, inputs, output):
            if self.step >= len(self.steps) or name not in self.steps[self.step]:
                return None
            ref = self.steps[self.step][name]
            out = output[0] if isinstance(output, tuple) else output
            if tuple(ref.shape) != tuple(out.shape):
                raise ValueError(f"replacement for {name} at step {self.step}: shape {tuple(ref.shape)} "
                                 f"!= output {tuple(out.shape)}")
            new = ref.to(device=out.device, dtype=out.dtype)
            self.replaced += 1
            return (new,) + tuple(output[1:]) if isinstance(output, tuple) else new
        return fn

    def next_step(self) -> None:
        self.step += 1

    def remove(self) -> None:
        for h in self.handles:
            h.remove()
        self.handles = []
