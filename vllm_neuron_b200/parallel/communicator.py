"""Device communicator: fused in-kernel NVLink collectives with NCCL as fallback.

Filled in by the symmetric-memory all-reduce; until a group has a communicator
attached every collective goes through NCCL.
"""

from __future__ import annotations


def attach_communicators(ps, device) -> None:
    return None
