"""Device communicator: fused in-kernel NVLink collectives, NCCL otherwise.

``FusedCommunicator`` owns one IPC-shared device region per rank of a group (see
``csrc/comm.cu``) and runs the one-shot all-reduce that is fused with the bias add,
residual add and RMSNorm which follow every all-reduce in the decoder.  It handles
bf16 activations up to ``max_tokens`` rows (decode and small prefill chunks); larger
tensors, other dtypes and CPU groups fall back to NCCL / gloo through the
``GroupCoordinator``.  ``SpCommunicator`` runs the sequence-parallel prefill boundary
(reduce-scatter + norm + all-gather in one kernel).  This is the B200 counterpart of the Trainium plugin's device
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
    CANARY_BYTES = 256
    CANARY_VALUE = 0xA5
    HEADER_BYTES = 64 * 1024  # flags + counters before the two slots (csrc/comm.cu)

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
        # LL protocol (data and epoch in every 16-byte store: no flag round trip, twice the
        # bytes); fixed for the communicator's life
        from .. import envs

        self.ll = 1 if envs.VLLM_B200_AR_LL else 0
        # one receive area per source rank in each of the two slots, each followed by a guard
        # of CANARY_BYTES that no kernel writes (a pattern checked by check_canaries)
        self.area_bytes = max_tokens * max_hidden * (4 if self.ll else 2)
        self.slot_bytes = group.world_size * (self.area_bytes + self.CANARY_BYTES)
        self.max_elems = max_tokens * max_hidden
        ops = torch.ops.b200
        with torch.cuda.device(device):
            self.local = ops.comm_alloc(self.slot_bytes)
            for off in self._canary_offsets():
                ops.device_fill(self.local + off, self.CANARY_BYTES, self.CANARY_VALUE)
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

    def _canary_offsets(self) -> list[int]:
        part = self.area_bytes + self.CANARY_BYTES
        return [self.HEADER_BYTES + slot * self.slot_bytes + p * part + self.area_bytes
                for slot in (0, 1) for p in range(self.world)]

    def check_canaries(self) -> bool:
        """Every guard after a receive area of this rank's region still holds its pattern (no
        kernel wrote past the rows it owns).  Synchronises the device."""
        ops = torch.ops.b200
        with torch.cuda.device(self.device):
            torch.cuda.synchronize()
            return all(bool((ops.device_read(self.local + off, self.CANARY_BYTES) == self.CANARY_VALUE).all())
                       for off in self._canary_offsets())

    def can_all_reduce(self, x: torch.Tensor) -> bool:
        return (x.is_cuda and x.dtype == torch.bfloat16 and x.is_contiguous() and x.dim() >= 1
                and x.shape[-1] % 8 == 0 and x.shape[-1] <= self.max_hidden and x.numel() <= self.max_elems)

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        out = torch.empty_like(x)
        torch.ops.b200.allreduce_fused(self.bases, self.rank, self.slot_bytes, x, out, None, None, None, 0.0,
                                       self.num_blocks, self.status, 0, None, 0, 0, self.ll)
        return out

    def all_reduce_routes_add_rmsnorm(self, y: torch.Tensor, topk_ids: torch.Tensor, e_local: int, e_off: int,
                                      residual: torch.Tensor, w: torch.Tensor, eps: float,
                                      bias: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        """The MoE layer boundary in one kernel: per token, the sum of its per-route expert
        rows ``y`` [T * k, H] over this rank's experts is the partial that is all-reduced, then
        bias, residual and RMSNorm as ``all_reduce_add_rmsnorm``."""
        T, H = topk_ids.shape[0], y.shape[-1]
        out = torch.empty(T, H, dtype=y.dtype, device=y.device)
        torch.ops.b200.allreduce_fused(self.bases, self.rank, self.slot_bytes, y, out, residual, bias, w, eps,
                                       self.num_blocks, self.status, 0, topk_ids, e_local, e_off, self.ll)
        return out, residual

    def all_reduce_add_rmsnorm(self, x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float,
                               bias: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        out = torch.empty_like(x)
        torch.ops.b200.allreduce_fused(self.bases, self.rank, self.slot_bytes, x, out, residual, bias, w, eps,
                                       self.num_blocks, self.status, 0, None, 0, 0, self.ll)
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


def _open_region(group, device, slot_bytes: int) -> tuple[int, list[int], list[int]]:
    """Allocate this rank's region (header + two slots of ``slot_bytes``) and map every peer's
    region through CUDA IPC: (local pointer, every rank's base in rank order, opened peers)."""
    ops = torch.ops.b200
    with torch.cuda.device(device):
        local = ops.comm_alloc(slot_bytes)
        handle = ops.ipc_get_handle(local).numpy().tobytes()
    handles = [None] * group.world_size
    dist.all_gather_object(handles, handle, group=group.cpu_group)
    bases, opened = [], []
    with torch.cuda.device(device):
        for p, h in enumerate(handles):
            if p == group.rank_in_group:
                bases.append(local)
            else:
                ptr = ops.ipc_open_handle(torch.frombuffer(bytearray(h), dtype=torch.uint8))
                bases.append(ptr)
                opened.append(ptr)
    return local, bases, opened


class SpCommunicator:
    """Sequence-parallel prefill layer boundaries over NVLink (``sp_boundary_kernel`` in
    ``csrc/comm.cu``).

    ``boundary`` replaces reduce-scatter + bias + residual add + RMSNorm + all-gather with one
    kernel of two push phases; its output ([T, H], every rank's normalised rows) is a view of
    this communicator's memory.  ``scatter_targets`` gives the row-parallel GEMM the addresses
    of the receive areas its partial rows belong in (``ops.linear_scatter``), so the
    reduce-scatter's data leaves tile by tile as the GEMM produces it and the boundary only
    reduces.  Each rank's region holds two slots of [RS areas | guard | AG area | guard]; the
    host alternates them per call (every rank makes the same calls), so an output stays valid
    until the call after next.  Reference: the SP boundaries of
    ``model/gpt_oss/model_mxfp4.py:464,685`` (all-gather before a block, reduce-scatter after)."""

    GUARD_BYTES = 256
    CANARY_VALUE = 0xA5
    HEADER_BYTES = 64 * 1024  # flags + counters (csrc/comm.cu)

    def __init__(self, group, device: torch.device, max_tokens: int, hidden: int, num_blocks: int = 128):
        from ..ops import _ext, device_status

        _ext.load()
        self.group = group
        self.device = device
        self.rank = group.rank_in_group
        self.world = group.world_size
        self.num_blocks = num_blocks
        self.hidden = hidden
        self.area_bytes = -(-max_tokens * hidden * 2 // 256) * 256
        self.slot_bytes = 2 * (self.area_bytes + self.GUARD_BYTES)
        self.calls = 0
        self.local, self.bases, self._opened = _open_region(group, device, self.slot_bytes)
        with torch.cuda.device(device):
            for off in self._canary_offsets():
                torch.ops.b200.device_fill(self.local + off, self.GUARD_BYTES, self.CANARY_VALUE)
        group.barrier()
        self.status = device_status(device)
        logger.info("SP communicator for group %s: %d ranks, %d rows x %d, %.1f MB", group.name, self.world,
                    max_tokens, hidden, 2 * self.slot_bytes / 1e6)

    def _canary_offsets(self) -> list[int]:
        a, g = self.area_bytes, self.GUARD_BYTES
        return [self.HEADER_BYTES + slot * self.slot_bytes + off for slot in (0, 1) for off in (a, 2 * a + g)]

    def check_canaries(self) -> bool:
        """Every guard of this rank's region still holds its pattern.  Synchronises the device."""
        ops = torch.ops.b200
        with torch.cuda.device(self.device):
            torch.cuda.synchronize()
            return all(bool((ops.device_read(self.local + off, self.GUARD_BYTES) == self.CANARY_VALUE).all())
                       for off in self._canary_offsets())

    def can(self, T: int, H: int) -> bool:
        return T > 0 and T % self.world == 0 and H % 8 == 0 and H <= 8192 and T * H * 2 <= self.area_bytes

    def scatter_targets(self, T: int, H: int) -> list[int]:
        """Where the next call's partial rows of this rank go: rank q's RS area for this source
        (rows q T / world .. of the partial), in the slot the next ``boundary`` call uses."""
        slot = self.calls & 1
        return [self.bases[q] + self.HEADER_BYTES + slot * self.slot_bytes + self.rank * (T // self.world) * H * 2
                for q in range(self.world)]

    def boundary(self, x: torch.Tensor | None, T: int, residual: torch.Tensor, w: torch.Tensor, eps: float,
                 bias: torch.Tensor | None = None, routes: tuple | None = None) -> torch.Tensor:
        """RMSNorm(reduce_scatter(x) + bias + residual) * w, all-gathered: [T, H] on every rank;
        ``residual`` (this rank's [T / world, H] rows) becomes the pre-norm sum.  ``x``: the
        [T, H] partial; with ``routes`` = (topk_ids, e_local, e_off) the [T * k, H] per-route
        expert rows of an MoE layer; None after ``ops.linear_scatter`` to ``scatter_targets``."""
        H = residual.shape[-1]
        slot = self.calls & 1
        self.calls += 1
        ids, e_local, e_off = routes if routes is not None else (None, 0, 0)
        torch.ops.b200.sp_boundary(self.bases, self.rank, self.slot_bytes, self.area_bytes, self.GUARD_BYTES, slot,
                                   x, residual, bias, w, eps, T, self.num_blocks, self.status, 0, ids, e_local, e_off)
        out = self.HEADER_BYTES + slot * self.slot_bytes + self.area_bytes + self.GUARD_BYTES
        return torch.ops.b200.comm_view(self.local + out, T, H, residual)

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


class NvlsReducer:
    """Row-parallel GEMM fused with the all-reduce, through NVSwitch multicast (NVLS).

    Owns one symmetric region per group (``torch.distributed._symmetric_memory`` allocates
    it and binds every rank's copy to a multicast object; the kernels are this library's).
    ``linear_add_rmsnorm`` runs two kernels (``csrc/gemm.cu``): the tcgen05 GEMM of this
    rank's K slice adds each fp32 output tile into the accumulator of every rank at once
    with ``multimem.red.add`` (the switch performs the additions) and counts the tile with a
    multicast release; the finish kernel waits for all ranks' tiles, then applies bias,
    residual and RMSNorm and clears the accumulator.  Decode-size token counts only
    (``max_tokens``).  This replaces GEMM -> all-reduce + RMSNorm at the reference's
    attention ``all_reduce`` (``model/gpt_oss/model_mxfp4.py:828``, ``nn/rpl.py:146-149``)."""

    def __init__(self, group, device: torch.device, max_tokens: int = 256, max_hidden: int = 8192,
                 max_splits: int = 8, num_blocks: int = 128):
        from torch.distributed import _symmetric_memory as symm

        from ..ops import _ext, device_status

        _ext.load()
        self.world = group.world_size
        self.T_cap, self.H_cap = max_tokens, max_hidden
        self.max_splits, self.num_blocks = max_splits, num_blocks
        nbytes = int(torch.ops.b200.red_region_bytes(max_tokens, max_hidden))
        gname = group.device_group.group_name
        try:
            symm.enable_symm_mem_for_group(gname)
        except Exception:  # noqa: BLE001  (newer torch: nothing to enable)
            pass
        with torch.cuda.device(device):
            self.buf = symm.empty(nbytes, dtype=torch.uint8, device=device)
            self.buf.zero_()
            self.hdl = symm.rendezvous(self.buf, gname)
        # the multicast address is used only when it provably maps this tensor: a handle at
        # offset 0 whose local buffer pointer is the tensor's own
        off = int(getattr(self.hdl, "offset", 0))
        ptrs = list(self.hdl.buffer_ptrs)
        mc = int(self.hdl.multicast_ptr or 0)
        if mc == 0 or off != 0 or int(ptrs[group.rank_in_group]) != self.buf.data_ptr():
            raise RuntimeError(f"no usable NVLS multicast mapping (mc={mc:#x}, offset={off})")
        self.uc, self.mc = self.buf.data_ptr(), mc
        self.status = device_status(device)
        torch.cuda.synchronize(device)
        group.barrier()
        logger.info("NVLS reducer for group %s: %d ranks, %.1f MB region", group.name, self.world, nbytes / 1e6)

    def can(self, x: torch.Tensor, weight: torch.Tensor) -> bool:
        T = x.numel() // x.shape[-1] if x.dim() else 0
        return (x.is_cuda and x.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16 and 0 < T <= self.T_cap
                and weight.shape[0] <= self.H_cap and weight.shape[0] % 8 == 0 and weight.shape[1] % 8 == 0
                and weight.is_contiguous())

    def linear_add_rmsnorm(self, x: torch.Tensor, weight: torch.Tensor, residual: torch.Tensor, w: torch.Tensor,
                           eps: float, bias: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        x2 = x.reshape(-1, x.shape[-1])
        if x2.stride(1) != 1 or x2.stride(0) % 8 or x2.data_ptr() % 16:
            x2 = x2.contiguous()
        ops = torch.ops.b200
        items = ops.gemm_bf16_allreduce(x2, weight, self.uc, self.mc, self.T_cap, self.H_cap, self.max_splits,
                                        self.status)
        out = torch.empty(x2.shape[0], weight.shape[0], dtype=x.dtype, device=x.device)
        bb = bias.to(torch.bfloat16).contiguous() if bias is not None else None
        ops.allreduce_finish(self.uc, self.T_cap, self.H_cap, items * self.world, out, residual, bb, w, eps,
                             self.num_blocks, self.status)
        return out, residual

    def close(self) -> None:
        self.hdl = None
        self.buf = None


def attach_reducers(ps, device) -> None:
    """NVLS GEMM + all-reduce for the TP group (collective: every rank calls it).  Groups
    without a usable multicast mapping keep the GEMM + fused all-reduce kernel pair."""
    from .. import envs

    if not envs.VLLM_B200_GEMM_ALLREDUCE:
        return
    seen = {}
    for name in ("tp", "attn_tp"):
        g = getattr(ps, name)
        if g.world_size <= 1 or g.world_size > 8 or g.device_group is None:
            continue
        key = tuple(g.ranks)
        if key not in seen:
            red, err = None, None
            try:
                red = NvlsReducer(g, device)
            except Exception as e:  # noqa: BLE001
                err = e
            # every rank of the group must take the same path: a rank waiting for tiles that a
            # rank on the other path never adds would only end by its wait limit
            ok = g.cpu_all_reduce_max([0 if red is not None else 1])[0] == 0
            if not ok:
                if red is not None:
                    red.close()
                red = None
                logger.warning("group %s: NVLS GEMM + all-reduce unavailable (%s); using GEMM + NVLink all-reduce",
                               g.name, err or "another rank has no multicast mapping")
            seen[key] = red
        g.reducer = seen[key]


def attach_sp_communicator(ps, device, max_tokens: int, hidden: int) -> None:
    """Give the TP group an ``SpCommunicator`` for prefill steps of up to ``max_tokens`` rows
    (capped at 16384) of ``hidden`` when sequence parallelism and its fused boundary
    (``VLLM_B200_FUSED_SP``) are on.  Collective."""
    from .. import envs

    g = ps.tp
    if (envs.VLLM_B200_SEQUENCE_PARALLEL and envs.VLLM_B200_FUSED_SP and 1 < g.world_size <= 8
            and g.device_group is not None):
        g.sp_comm = SpCommunicator(g, device, min(max_tokens, 16384), hidden)


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
