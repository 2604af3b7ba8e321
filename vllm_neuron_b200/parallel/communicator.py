"""Device communicator: fused in-kernel NVLink collectives, NCCL otherwise.

``FusedCommunicator`` owns one IPC-shared device region per rank of a group (see
``csrc/comm.cu``) and runs the one-shot all-reduce that is fused with the bias add,
residual add and RMSNorm which follow every all-reduce in the decoder.  It handles
bf16 activations up to ``max_tokens`` rows (decode and small prefill chunks); larger
tensors, other dtypes and CPU groups fall back to NCCL / gloo through the
``GroupCoordinator``.  This is the B200 counterpart of the Trainium plugin's device
communicator (``vllm_neuron/parallel/neuron_communicator.py:13``), whose collectives
were XLA HLO ops.

Every call on one communicator launches the same fixed number of CTAs; the kernel's
per-CTA epochs and double-buffered slots rely on it.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..logging_config import init_logger

logger = init_logger(__name__)


class FusedCommunicator:
    def __init__(self, group, device: torch.device, max_tokens: int = 256, max_hidden: int = 8192,
                 num_blocks: int = 64):
        from ..ops import _ext

        _ext.load()
        self.group = group
        self.device = device
        self.rank = group.rank_in_group
        self.world = group.world_size
        self.num_blocks = num_blocks
        self.max_hidden = max_hidden
        # one receive area per source rank in each of the two slots
        self.slot_bytes = group.world_size * max_tokens * max_hidden * 2
        self.max_elems = max_tokens * max_hidden
        ops = torch.ops.b200
        with torch.cuda.device(device):
            self.local = ops.comm_alloc(self.slot_bytes)
            handle = ops.ipc_get_handle(self.local).numpy().tobytes()
        handles = [None] * self.world
        dist.all_gather_object(handles, handle, group=group.cpu_group)
        self.bases: list[int] = []
        self._opened: list[int] = []
        with torch.cuda.device(device):
            for p, h in enumerate(handles):
                if p == self.rank:
                    self.bases.append(self.local)
                else:
                    ptr = ops.ipc_open_handle(torch.frombuffer(bytearray(h), dtype=torch.uint8))
                    self.bases.append(ptr)
                    self._opened.append(ptr)
        group.barrier()
        from ..ops import device_status

        self.status = device_status(device)
        logger.info("fused communicator for group %s: %d ranks, %.1f MB slots", group.name, self.world,
                    self.slot_bytes / 1e6)

    def can_all_reduce(self, x: torch.Tensor) -> bool:
        return (x.is_cuda and x.dtype == torch.bfloat16 and x.is_contiguous() and x.dim() >= 1
                and x.shape[-1] % 8 == 0 and x.shape[-1] <= self.max_hidden and x.numel() <= self.max_elems)

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        out = torch.empty_like(x)
        torch.ops.b200.allreduce_fused(self.bases, self.rank, self.slot_bytes, x, out, None, None, None, 0.0,
                                       self.num_blocks, self.status)
        return out

    def all_reduce_add_rmsnorm(self, x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float,
                               bias: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        out = torch.empty_like(x)
        torch.ops.b200.allreduce_fused(self.bases, self.rank, self.slot_bytes, x, out, residual, bias, w, eps,
                                       self.num_blocks, self.status)
        return out, residual

    def close(self) -> None:
        ops = torch.ops.b200
        try:
            torch.cuda.synchronize(self.device)
            for p in self._opened:
                ops.ipc_close(p)
            ops.comm_free(self.local)
        except Exception:  # noqa: BLE001
            pass
        self._opened = []


def attach_communicators(ps, device) -> None:
    """Create fused communicators for the groups whose all-reduces sit on the decode hot
    path (TP, and the MoE group when it differs).  Collective: every rank calls it."""
    seen = {}
    for name in ("tp", "moe", "world", "attn_tp"):
        g = getattr(ps, name)
        if g.world_size <= 1 or g.world_size > 8:
            continue
        key = tuple(g.ranks)
        if key not in seen:
            seen[key] = FusedCommunicator(g, device)
        g.communicator = seen[key]
