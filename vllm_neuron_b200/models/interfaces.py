"""Optional model capabilities, checked with ``isinstance`` (the reference's
``model/interfaces.py``: ``SupportsVisionWarmup`` ``:14``, ``SupportsSpatialMerge`` ``:28``,
``SupportsMaxPixels`` ``:38``, ``SupportsMRoPE`` ``:63``).

* ``SupportsVisionWarmup``: builds vision-encoder inputs that produce exactly ``bucket``
  merged tokens, so the worker can run the encoder once per configured size at start-up.
* ``SupportsSpatialMerge``: how many raw patches collapse into one embedding token.
* ``SupportsMaxPixels``: the raw patch count of an image at a pixel budget.
* ``SupportsMRoPE``: 3-D rotary positions of a prompt with expanded image placeholders.
"""

from __future__ import annotations

from typing import Protocol, runtime_checkable

import torch


@runtime_checkable
class SupportsVisionWarmup(Protocol):
    def build_vision_synthetic_inputs(self, bucket: int, vision_neuron_config, device: torch.device) -> dict:
        ...


@runtime_checkable
class SupportsSpatialMerge(Protocol):
    @classmethod
    def get_vision_token_merge_factor(cls, hf_config) -> int:
        ...


@runtime_checkable
class SupportsMaxPixels(Protocol):
    @classmethod
    def get_max_pixels_token_count(cls, hf_config, max_pixels: int) -> int:
        ...


@runtime_checkable
class SupportsMRoPE(Protocol):
    def get_mrope_input_positions(self, token_ids: list[int], grids: list) -> tuple[torch.Tensor, int]:
        ...


def _vision_cfg(hf_config) -> dict:
    """The vision sub-config of an HF config given as a dict or a PretrainedConfig."""
    if isinstance(hf_config, dict):
        return dict(hf_config.get("vision_config") or {})
    v = getattr(hf_config, "vision_config", None)
    return v.to_dict() if hasattr(v, "to_dict") else dict(vars(v)) if v is not None else {}
