"""Process groups for every parallelism the framework supports.

One process per GPU.  This module owns every group, the same set the Trainium
plugin builds in ``vllm_neuron/parallel/neuron_parallel_state.py:51-91,328-662``:
TP, DP, EP and EP-TP (variable EP), attention-DP columns and attention-TP
supergroups, component-DP supergroups (embedding / lm_head / mlp), decode context
parallel (DCP) groups, sampling-DP meshes and vision TP/DP.

Differences, by design:
* Ranks are laid out contiguously (rank = dp_index * tp + tp_index).  NVSwitch gives
  every GPU the same bandwidth to every peer, so the Trn2 8x8 torus remap
  (``neuron_parallel_state.py:133-143``) has no equivalent.
* Each group carries a device group (NCCL on GPU, gloo on CPU) and a CPU gloo group
  for control-plane traffic (DP padding MAX-reduce, barriers, object broadcast).
* Device collectives go through :class:`GroupCoordinator`, which dispatches to the
  fused NVLink kernels of :mod:`vllm_neuron_b200.parallel.communicator` when they
  are available and to NCCL otherwise.

The rank-list builders are pure functions so they are unit-tested without any
process group.
"""

from __future__ import annotations

import datetime
import os
from dataclasses import dataclass, field
from typing import Any

import torch
import torch.distributed as dist

from ..logging_config import init_logger

logger = init_logger(__name__)


# ---------------------------------------------------------------------------
# Pure rank math
# ---------------------------------------------------------------------------


def build_2d_mesh(ranks: list[int], row_size: int, num_rows: int) -> tuple[list[list[int]], list[list[int]]]:
    """Row groups are contiguous runs of ``row_size`` ranks; column groups take the
    same position of every row."""
    if row_size * num_rows != len(ranks):
        raise ValueError(f"mesh {num_rows}x{row_size} does not cover {len(ranks)} ranks")
    rows = [ranks[i * row_size:(i + 1) * row_size] for i in range(num_rows)]
    cols = [[rows[r][c] for r in range(num_rows)] for c in range(row_size)]
    return rows, cols


def build_tp_dp_group_ranks(world_size: int, tp: int) -> tuple[list[list[int]], list[list[int]]]:
    """TP groups (rows) and DP groups (columns)."""
    if world_size % tp:
        raise ValueError(f"world size {world_size} not divisible by tp {tp}")
    return build_2d_mesh(list(range(world_size)), tp, world_size // tp)


def build_ep_group_ranks(world_size: int, ep_degree: int) -> tuple[list[list[int]], list[list[int]]]:
    """(EP-TP rows, EP columns).  Each EP partition owns ``E/ep`` experts and shards
    their intermediate dimension over its ``world/ep`` EP-TP ranks."""
    if world_size % ep_degree:
        raise ValueError(f"world size {world_size} not divisible by ep_degree {ep_degree}")
    return build_2d_mesh(list(range(world_size)), world_size // ep_degree, ep_degree)


def build_sampling_dp_meshes(tp: int, dp: int) -> tuple[list[list[int]], list[list[int]]]:
    """(all2all groups of ``dp`` ranks, gather groups = transpose)."""
    if tp % dp:
        raise ValueError(f"tp ({tp}) must be divisible by sampling_dp_degree ({dp})")
    return build_2d_mesh(list(range(tp)), dp, tp // dp)


def build_component_tp_group_ranks(world_size: int, tp: int, dp_component: int) -> list[list[int]]:
    """Supergroups of ``tp * dp_component`` ranks: DP0's TP ranks, then DP1's, ..."""
    dp = world_size // tp
    if dp % dp_component:
        raise ValueError(f"dp_size ({dp}) must be divisible by dp_component_size ({dp_component})")
    out = []
    for sg in range(dp // dp_component):
        out.append([(sg * dp_component + d) * tp + t for d in range(dp_component) for t in range(tp)])
    return out


def build_component_dp_group_ranks(world_size: int, tp: int, dp_component: int) -> list[list[int]]:
    """Inside every component supergroup, the ranks at the same TP position (one per DP
    replica of the supergroup): the group over which a component-DP module gathers its
    input rows (``model_mxfp4.py:1484-1501`` transitions between these states)."""
    out = []
    for sg in build_component_tp_group_ranks(world_size, tp, dp_component):
        for t in range(tp):
            out.append([sg[d * tp + t] for d in range(dp_component)])
    return out


def build_dp_column_group_ranks(world_size: int, tp: int, attention_dp: int) -> list[list[int]]:
    """Attention-DP columns: same TP position across ``attention_dp`` consecutive DP replicas."""
    dp = world_size // tp
    if dp % attention_dp:
        raise ValueError(f"dp_size ({dp}) must be divisible by attention_dp_size ({attention_dp})")
    out = []
    for sg in range(dp // attention_dp):
        for t in range(tp):
            out.append([(sg * attention_dp + d) * tp + t for d in range(attention_dp)])
    return out


def build_dcp_group_ranks(world_size: int, tp: int, dcp: int) -> tuple[list[list[int]], list[list[int]]]:
    """Decode context parallel.  KV groups are runs of ``dcp`` consecutive ranks of a TP
    group: TP shards KV heads contiguously (rank r holds head r // (tp / kv_heads) when
    TP exceeds the head count), so consecutive ranks hold the same KV head and split its
    tokens.  Head groups take one rank from each run (stride ``dcp``) and shard the heads.
    The reference strides its KV groups instead (``neuron_parallel_state.py:361-414``)
    because it also re-orders the head sharding under DCP; here the TP sharding is kept."""
    if tp % dcp:
        raise ValueError(f"dcp ({dcp}) must divide tp ({tp})")
    kv_groups, head_groups = [], []
    for base in range(0, world_size, tp):
        ranks = list(range(base, base + tp))
        rows, cols = build_2d_mesh(ranks, dcp, tp // dcp)
        kv_groups.extend(rows)
        head_groups.extend(cols)
    return kv_groups, head_groups


def build_inter_node_peer_group_ranks(world_size: int, nnodes: int) -> list[list[int]]:
    if world_size % nnodes:
        raise ValueError(f"world_size ({world_size}) must be divisible by nnodes ({nnodes})")
    per = world_size // nnodes
    return [[n * per + p for n in range(nnodes)] for p in range(per)]


def node_of(rank: int, world_size: int, nnodes: int) -> int:
    return rank // (world_size // nnodes)


# ---------------------------------------------------------------------------
# Group coordinator
# ---------------------------------------------------------------------------


@dataclass
class RoutePartial:
    """An MoE layer's output before its per-token route sum: ``y`` [T * k, H] per-route
    expert rows (the routes to this rank's experts [e_off, e_off + e_local) written), summed
    by the layer-boundary all-reduce kernel itself; ``materialize`` sums them here."""
    y: torch.Tensor
    topk_ids: torch.Tensor
    e_local: int
    e_off: int

    @property
    def shape(self) -> torch.Size:
        return torch.Size((self.topk_ids.shape[0], self.y.shape[-1]))

    def materialize(self) -> torch.Tensor:
        out = torch.empty(self.shape, dtype=self.y.dtype, device=self.y.device)
        torch.ops.b200.moe_route_sum(out, self.y, self.topk_ids, self.e_local, self.e_off)
        return out


@dataclass
class GroupCoordinator:
    """A device group plus a CPU group over the same ranks."""

    name: str
    ranks: list[int]
    device_group: Any = None
    cpu_group: Any = None
    rank: int = 0
    communicator: Any = None  # fused NVLink collectives (parallel.communicator)
    reducer: Any = None  # GEMM fused with the all-reduce through NVSwitch (parallel.communicator)
    sp_comm: Any = None  # sequence-parallel prefill boundary over NVLink (parallel.communicator)
    sp_active: bool = False  # sequence parallelism at layer boundaries (set per prefill step)

    @property
    def world_size(self) -> int:
        return len(self.ranks)

    @property
    def rank_in_group(self) -> int:
        return self.ranks.index(self.rank)

    @property
    def is_first_rank(self) -> bool:
        return self.rank_in_group == 0

    # -- device collectives -------------------------------------------------
    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        if self.world_size == 1:
            return x
        if self.communicator is not None and self.communicator.can_all_reduce(x):
            return self.communicator.all_reduce(x)
        dist.all_reduce(x, group=self.device_group)
        return x

    def all_reduce_add_rmsnorm(self, x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float,
                               bias: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        """(RMSNorm(sum_ranks(x) + bias + residual) * w, sum + bias + residual).  One fused
        NVLink kernel when a communicator can take ``x``; otherwise all-reduce then the
        fused add+norm op."""
        from .. import ops

        if isinstance(x, RoutePartial):
            comm = self.communicator
            T = x.shape[0]
            if self.sp_active and self.world_size > 1 and self.sp_comm is not None and self.sp_comm.can(T, x.shape[1]):
                return self._sp_boundary(x.y, T, residual, w, eps, bias, (x.topk_ids, x.e_local, x.e_off))
            if (self.world_size > 1 and comm is not None and not self.sp_active
                    and comm.can_all_reduce(residual)):
                return comm.all_reduce_routes_add_rmsnorm(x.y, x.topk_ids, x.e_local, x.e_off, residual, w, eps, bias)
            x = x.materialize()
        if self.sp_active and self.world_size > 1 and x.shape[0] % self.world_size == 0:
            return self._sp_add_rmsnorm(x, residual, w, eps, bias)
        if self.world_size > 1 and self.communicator is not None and self.communicator.can_all_reduce(x):
            return self.communicator.all_reduce_add_rmsnorm(x, residual, w, eps, bias)
        if self.world_size > 1:
            x = self.all_reduce(x)
        if bias is not None:
            x = x + bias
        return ops.fused_add_rms_norm(x, residual, w, eps)

    def linear_all_reduce_add_rmsnorm(self, x: torch.Tensor, weight: torch.Tensor, residual: torch.Tensor,
                                      w: torch.Tensor, eps: float, bias: torch.Tensor | None = None
                                      ) -> tuple[torch.Tensor, torch.Tensor]:
        """Row-parallel projection and layer boundary: (RMSNorm(sum_ranks(x . weight^T) + bias
        + residual) * w, the new residual).  With an NVLS reducer the GEMM's output tiles are
        reduced through NVSwitch by the GEMM itself and one small kernel normalises; otherwise
        the GEMM runs, then :meth:`all_reduce_add_rmsnorm`."""
        from .. import ops

        if (self.world_size > 1 and not self.sp_active and self.reducer is not None
                and self.reducer.can(x, weight)):
            return self.reducer.linear_add_rmsnorm(x, weight, residual, w, eps, bias)
        sc = self.sp_comm
        T = x.shape[0] if x.dim() == 2 else -1
        if (self.sp_active and self.world_size > 1 and sc is not None and sc.can(T, weight.shape[0])
                and ops.gemm_available(x, weight)):
            # GEMM -> reduce-scatter fused: the GEMM stores each partial row block in its
            # owner's receive area; the boundary kernel reduces, normalises and all-gathers
            ops.linear_scatter(x, weight, sc.scatter_targets(T, weight.shape[0]), weight.shape[0])
            return self._sp_boundary(None, T, residual, w, eps, bias)
        return self.all_reduce_add_rmsnorm(ops.linear(x, weight, None), residual, w, eps, bias)

    def _sp_boundary(self, x, T, residual, w, eps, bias, routes=None):
        """The SP boundary in one NVLink kernel (``SpCommunicator.boundary``); the residual
        becomes this rank's T / tp rows at the first boundary."""
        if residual.shape[0] == T:  # first boundary after the (replicated) embedding
            residual = residual.chunk(self.world_size, dim=0)[self.rank_in_group].contiguous()
        return self.sp_comm.boundary(x, T, residual, w, eps, bias, routes), residual

    def _sp_add_rmsnorm(self, x, residual, w, eps, bias):
        """Sequence-parallel layer boundary (prefill): reduce-scatter the partial sums over
        tokens, add bias and this rank's residual rows, normalise the shard, all-gather the
        normalised rows for the next GEMM.  The residual stays sharded (T / tp rows)
        between boundaries (``model_mxfp4.py:464,685``: AG before, RS after each block).
        One NVLink kernel when an ``SpCommunicator`` is attached, else NCCL + the norm."""
        from .. import ops

        T = x.shape[0]
        if self.sp_comm is not None and x.is_cuda and x.dtype == torch.bfloat16 and self.sp_comm.can(T, x.shape[-1]):
            return self._sp_boundary(x.contiguous(), T, residual, w, eps, bias)
        xs = self.reduce_scatter(x, dim=0)
        if residual.shape[0] == T:  # first boundary after the (replicated) embedding
            residual = residual.chunk(self.world_size, dim=0)[self.rank_in_group].contiguous()
        if bias is not None:
            xs = xs + bias
        y, r = ops.fused_add_rms_norm(xs, residual, w, eps)
        return self.all_gather(y, dim=0), r

    def all_gather(self, x: torch.Tensor, dim: int = 0) -> torch.Tensor:
        if self.world_size == 1:
            return x
        if dim < 0:
            dim += x.dim()
        xc = x.movedim(dim, 0).contiguous()
        out = torch.empty((self.world_size * xc.shape[0],) + tuple(xc.shape[1:]), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(out, xc, group=self.device_group)
        return out.movedim(0, dim)

    def reduce_scatter(self, x: torch.Tensor, dim: int = 0) -> torch.Tensor:
        if self.world_size == 1:
            return x
        if dim < 0:
            dim += x.dim()
        xc = x.movedim(dim, 0).contiguous()
        if xc.shape[0] % self.world_size:
            raise ValueError(f"reduce_scatter dim {xc.shape[0]} not divisible by {self.world_size}")
        out = torch.empty((xc.shape[0] // self.world_size,) + tuple(xc.shape[1:]), dtype=x.dtype, device=x.device)
        dist.reduce_scatter_tensor(out, xc, group=self.device_group)
        return out.movedim(0, dim)

    def all_to_all(self, x: torch.Tensor, scatter_dim: int = 0, gather_dim: int = 0) -> torch.Tensor:
        """Split ``x`` along ``scatter_dim`` into world chunks, exchange, concat along
        ``gather_dim`` (``functional/collectives/all_to_all.py:12``)."""
        if self.world_size == 1:
            return x
        if x.shape[scatter_dim] % self.world_size:
            raise ValueError(f"all_to_all dim {x.shape[scatter_dim]} not divisible by {self.world_size}")
        send = torch.stack(torch.chunk(x, self.world_size, dim=scatter_dim)).contiguous()
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=self.device_group)
        return torch.cat(list(recv.unbind(0)), dim=gather_dim)

    def all_to_all_v(self, x: torch.Tensor, send_counts: list[int], recv_counts: list[int]) -> torch.Tensor:
        if self.world_size == 1:
            return x
        out = torch.empty((sum(recv_counts),) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
        dist.all_to_all_single(out, x.contiguous(), recv_counts, send_counts, group=self.device_group)
        return out

    def broadcast(self, x: torch.Tensor, src_in_group: int = 0) -> torch.Tensor:
        if self.world_size > 1:
            dist.broadcast(x, self.ranks[src_in_group], group=self.device_group)
        return x

    # -- CPU control plane ---------------------------------------------------
    def broadcast_object(self, obj: Any = None, src_in_group: int = 0) -> Any:
        if self.world_size == 1:
            return obj
        lst = [obj]
        dist.broadcast_object_list(lst, src=self.ranks[src_in_group], group=self.cpu_group)
        return lst[0]

    def all_gather_object(self, obj: Any) -> list:
        if self.world_size == 1:
            return [obj]
        out: list = [None] * self.world_size
        dist.all_gather_object(out, obj, group=self.cpu_group)
        return out

    def cpu_all_reduce_max(self, values: list[int]) -> list[int]:
        if self.world_size == 1:
            return list(values)
        t = torch.tensor(values, dtype=torch.int64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.cpu_group)
        return t.tolist()

    def lockstep_all_reduce_max(self, values: list[int], step: int, tag: int) -> list[int]:
        """``cpu_all_reduce_max`` that also proves every rank is at the same ``step`` and the
        same call site (``tag``): both ride along as (x, -x) pairs, whose MAX-reduce gives the
        largest and the smallest value.  A rank that skipped or repeated a step, or reached a
        different reduce, makes every rank raise instead of silently mixing one call's values
        with another's (the reference's data-parallel padding tripwire,
        ``neuron_model_runner.py:2765-2791``)."""
        out = self.cpu_all_reduce_max([step, -step, tag, -tag] + list(values))
        if out[0] != -out[1] or out[2] != -out[3]:
            raise RuntimeError(f"lockstep violated on rank {self.rank_in_group}: steps {-out[1]}..{out[0]}, "
                               f"call sites {-out[3]}..{out[2]} (this rank: step {step}, site {tag})")
        return out[4:]

    def barrier(self, timeout_s: float | None = None) -> None:
        """Barrier on the CPU group with a timeout (``neuron_parallel_state.py:1289-1325``)."""
        if self.world_size == 1:
            return
        if timeout_s is not None and hasattr(dist, "monitored_barrier"):
            try:
                dist.monitored_barrier(group=self.cpu_group, timeout=datetime.timedelta(seconds=timeout_s))
                return
            except RuntimeError as e:  # noqa: PERF203
                if "monitored_barrier" in str(e) and "not supported" in str(e):
                    pass
                else:
                    raise
        dist.barrier(group=self.cpu_group)


@dataclass
class ParallelState:
    world: GroupCoordinator
    tp: GroupCoordinator
    dp: GroupCoordinator
    ep: GroupCoordinator
    ep_tp: GroupCoordinator
    moe: GroupCoordinator  # group whose all-reduce completes the MoE output
    attn_tp: GroupCoordinator
    attn_dp: GroupCoordinator
    dcp_kv: GroupCoordinator
    dcp_head: GroupCoordinator
    embedding: GroupCoordinator
    lm_head: GroupCoordinator
    mlp: GroupCoordinator
    vision_tp: GroupCoordinator
    vision_dp: GroupCoordinator
    degrees: dict = field(default_factory=dict)
    # sampling DP within each TP group: all-to-all groups of ``sampling_dp`` consecutive
    # ranks (batch <-> vocab) and gather groups across them (``neuron_parallel_state.py:
    # 170-187,464-492``)
    sampling_a2a: GroupCoordinator | None = None
    sampling_gather: GroupCoordinator | None = None
    # component DP: the DP ranks of an embedding / lm_head / mlp supergroup
    embedding_dp: GroupCoordinator | None = None
    lm_head_dp: GroupCoordinator | None = None
    mlp_dp: GroupCoordinator | None = None
    # multi-node jobs: the ranks of this node, and the ranks at this rank's local position on
    # every node (``_build_inter_node_positional_peer_group_ranks``,
    # ``neuron_parallel_state.py:280``); both None on one node
    nnodes: int = 1
    node: GroupCoordinator | None = None
    inter_node: GroupCoordinator | None = None

    def component(self, name: str) -> tuple[GroupCoordinator, GroupCoordinator | None]:
        """(sharding group, DP gather group or None) of the "embedding", "lm_head" or "mlp"
        component: the TP group unless its component-DP degree is above 1."""
        dp_g = getattr(self, name + "_dp")
        if dp_g is None or dp_g.world_size == 1:
            return self.tp, None
        return getattr(self, name), dp_g


_STATE: ParallelState | None = None
_ALL_PGS: list[Any] = []


def _single(name: str, rank: int = 0) -> GroupCoordinator:
    return GroupCoordinator(name=name, ranks=[rank], rank=rank)


def _new_groups(name: str, rank_lists: list[list[int]], rank: int, backend: str,
                timeout: datetime.timedelta) -> GroupCoordinator:
    """Every rank must call new_group for every list, in the same order."""
    mine = None
    for ranks in rank_lists:
        if len(ranks) == 1:
            dev = cpu = None
        else:
            dev = dist.new_group(ranks, backend=backend, timeout=timeout)
            cpu = dist.new_group(ranks, backend="gloo", timeout=timeout) if backend != "gloo" else dev
            _ALL_PGS.extend([dev, cpu])
        if rank in ranks:
            mine = GroupCoordinator(name=name, ranks=list(ranks), device_group=dev, cpu_group=cpu, rank=rank)
    if mine is None:
        raise RuntimeError(f"rank {rank} not in any {name} group")
    return mine


def init_distributed_environment(world_size: int = 1, rank: int = 0, backend: str | None = None,
                                 init_method: str | None = None, local_rank: int = 0,
                                 timeout_s: float = 1800.0) -> None:
    """Create the default process group if needed (rendezvous on 127.0.0.1 by default)."""
    if world_size <= 1 or dist.is_initialized():
        return
    from .. import envs

    backend = backend or envs.get_dist_backend()
    if init_method is None:
        from ..utils.rendezvous import init_method_from_env

        init_method = init_method_from_env()  # file store of ranks spawned on this host
    if init_method is None:
        validate_master_addr(world_size)
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29533")
        init_method = "env://"
    if backend == "nccl":
        torch.cuda.set_device(local_rank)
    kw = dict(backend=backend, init_method=init_method, world_size=world_size, rank=rank,
              timeout=datetime.timedelta(seconds=timeout_s))
    if backend == "nccl":
        kw["device_id"] = torch.device("cuda", local_rank)
    dist.init_process_group(**kw)


_LOOPBACK = ("127.0.0.1", "localhost", "::1", "0.0.0.0")


def validate_master_addr(world_size: int, init_method: str | None = None) -> None:
    """A job spread over several nodes cannot rendezvous on a loopback address: the ranks of
    the other nodes would each wait on their own host until the timeout.  Raise a clear error
    instead (``validate_cross_node_master_addr``, ``vllm/worker/neuron_worker.py:56``).  Only
    ``env://`` rendezvous is checked; the nodes come from ``LOCAL_WORLD_SIZE``."""
    if _default_nnodes(world_size) <= 1:
        return
    if init_method not in (None, "env://"):
        return
    addr = os.environ.get("MASTER_ADDR", "127.0.0.1")
    if addr in _LOOPBACK:
        raise ValueError(f"{_default_nnodes(world_size)} nodes ({world_size} ranks, LOCAL_WORLD_SIZE="
                         f"{os.environ.get('LOCAL_WORLD_SIZE')}) but MASTER_ADDR={addr!r} is a loopback address; "
                         "set MASTER_ADDR (torchrun --master-addr / --rdzv-endpoint) to the head node's address "
                         "on every node")


def build_node_group_ranks(world_size: int, nnodes: int) -> tuple[list[list[int]], list[list[int]]]:
    """(ranks of each node, positional peers): ranks are dealt to nodes in contiguous blocks;
    peer group l holds local position l of every node."""
    if nnodes < 1 or world_size % nnodes:
        raise ValueError(f"world size {world_size} not divisible by nnodes {nnodes}")
    per = world_size // nnodes
    return ([[n * per + l for l in range(per)] for n in range(nnodes)],
            [[n * per + l for n in range(nnodes)] for l in range(per)])


def _default_nnodes(world_size: int) -> int:
    """Nodes of a torchrun job (``LOCAL_WORLD_SIZE`` ranks per node), else one."""
    local = int(os.environ.get("LOCAL_WORLD_SIZE", "0") or 0)
    return world_size // local if local > 0 and world_size % local == 0 else 1


def initialize_parallel_state(tp: int = 1, dp: int = 1, ep_degree: int = 1, attention_dp_size: int = 1,
                              embedding_dp_size: int = 1, lm_head_dp_size: int = 1, mlp_dp_size: int = 1,
                              dcp: int = 1, vision_tp: int | None = None, vision_dp: int | None = None,
                              backend: str | None = None, timeout_s: float = 1800.0,
                              sampling_dp: int = 1, nnodes: int | None = None) -> ParallelState:
    """Build every group (``initialize_neuron_parallel_state``, ``neuron_parallel_state.py:863``)."""
    global _STATE
    from .. import envs

    world_size = dist.get_world_size() if dist.is_initialized() else 1
    rank = dist.get_rank() if dist.is_initialized() else 0
    if tp * dp != world_size:
        raise ValueError(f"tp({tp}) x dp({dp}) != world size {world_size}")
    if world_size % ep_degree:
        raise ValueError(f"world size {world_size} not divisible by ep_degree {ep_degree}")
    vtp, vdp = vision_tp, vision_dp
    if vtp is None and vdp is None:
        vtp, vdp = tp, world_size // tp
    elif vtp is None:
        vtp = world_size // vdp
    elif vdp is None:
        vdp = world_size // vtp
    if vtp * vdp != world_size:
        raise ValueError(f"vision tp({vtp}) x dp({vdp}) != world size {world_size}")

    degrees = dict(world=world_size, tp=tp, dp=dp, ep=ep_degree, attention_dp=attention_dp_size,
                   embedding_dp=embedding_dp_size, lm_head_dp=lm_head_dp_size, mlp_dp=mlp_dp_size,
                   dcp=dcp, vision_tp=vtp, vision_dp=vdp, sampling_dp=sampling_dp)
    if world_size == 1:
        g = {k: _single(k) for k in ("world", "tp", "dp", "ep", "ep_tp", "moe", "attn_tp", "attn_dp", "dcp_kv",
                                     "dcp_head", "embedding", "lm_head", "mlp", "vision_tp", "vision_dp",
                                     "sampling_a2a", "sampling_gather", "embedding_dp", "lm_head_dp", "mlp_dp")}
        _STATE = ParallelState(**g, degrees=degrees)
        return _STATE

    backend = backend or envs.get_dist_backend()
    to = datetime.timedelta(seconds=timeout_s)
    tp_rows, dp_cols = build_tp_dp_group_ranks(world_size, tp)
    eptp_rows, ep_cols = build_ep_group_ranks(world_size, ep_degree)
    world_g = _new_groups("world", [list(range(world_size))], rank, backend, to)
    tp_g = _new_groups("tp", tp_rows, rank, backend, to)
    dp_g = _new_groups("dp", dp_cols, rank, backend, to)
    ep_g = _new_groups("ep", ep_cols, rank, backend, to)
    eptp_g = _new_groups("ep_tp", eptp_rows, rank, backend, to)
    attn_dp_g = _new_groups("attn_dp", build_dp_column_group_ranks(world_size, tp, attention_dp_size), rank,
                            backend, to)
    attn_tp_g = _new_groups("attn_tp", build_component_tp_group_ranks(world_size, tp, attention_dp_size), rank,
                            backend, to)
    emb_g = _new_groups("embedding", build_component_tp_group_ranks(world_size, tp, embedding_dp_size), rank,
                        backend, to)
    lmh_g = _new_groups("lm_head", build_component_tp_group_ranks(world_size, tp, lm_head_dp_size), rank,
                        backend, to)
    mlp_g = _new_groups("mlp", build_component_tp_group_ranks(world_size, tp, mlp_dp_size), rank, backend, to)
    emb_dp_g = _new_groups("embedding_dp", build_component_dp_group_ranks(world_size, tp, embedding_dp_size), rank,
                           backend, to)
    lmh_dp_g = _new_groups("lm_head_dp", build_component_dp_group_ranks(world_size, tp, lm_head_dp_size), rank,
                           backend, to)
    mlp_dp_g = _new_groups("mlp_dp", build_component_dp_group_ranks(world_size, tp, mlp_dp_size), rank, backend,
                           to)
    kv_rows, head_rows = build_dcp_group_ranks(world_size, tp, dcp)
    dcp_kv_g = _new_groups("dcp_kv", kv_rows, rank, backend, to)
    dcp_head_g = _new_groups("dcp_head", head_rows, rank, backend, to)
    vtp_rows, vdp_cols = build_2d_mesh(list(range(world_size)), vtp, vdp)
    vtp_g = _new_groups("vision_tp", vtp_rows, rank, backend, to)
    vdp_g = _new_groups("vision_dp", vdp_cols, rank, backend, to)
    s_rows, s_cols = build_sampling_dp_meshes(tp, sampling_dp)
    bases = range(0, world_size, tp)
    sa2a_g = _new_groups("sampling_a2a", [[b + r for r in row] for b in bases for row in s_rows], rank, backend, to)
    sgat_g = _new_groups("sampling_gather", [[b + r for r in col] for b in bases for col in s_cols], rank, backend,
                         to)
    # With EP the MoE output is completed by an all-reduce over every rank that
    # holds a slice of the experts for these tokens: the whole world when the
    # tokens are replicated across DP (wide EP), else the TP group.
    moe_g = world_g if ep_degree > 1 else mlp_g
    nn = nnodes if nnodes is not None else _default_nnodes(world_size)
    node_g = inter_g = None
    if nn > 1:
        node_rows, peer_rows = build_node_group_ranks(world_size, nn)
        node_g = _new_groups("node", node_rows, rank, backend, to)
        inter_g = _new_groups("inter_node", peer_rows, rank, backend, to)
    degrees["nnodes"] = nn
    _STATE = ParallelState(world=world_g, tp=tp_g, dp=dp_g, ep=ep_g, ep_tp=eptp_g, moe=moe_g, attn_tp=attn_tp_g,
                           attn_dp=attn_dp_g, dcp_kv=dcp_kv_g, dcp_head=dcp_head_g, embedding=emb_g,
                           lm_head=lmh_g, mlp=mlp_g, vision_tp=vtp_g, vision_dp=vdp_g, degrees=degrees,
                           sampling_a2a=sa2a_g, sampling_gather=sgat_g, embedding_dp=emb_dp_g,
                           lm_head_dp=lmh_dp_g, mlp_dp=mlp_dp_g, nnodes=nn, node=node_g, inter_node=inter_g)
    logger.info("parallel state: %s", degrees)
    return _STATE


def get_parallel_state() -> ParallelState:
    if _STATE is None:
        return initialize_parallel_state()
    return _STATE


def parallel_state_initialized() -> bool:
    return _STATE is not None


def get_tp_group() -> GroupCoordinator:
    return get_parallel_state().tp


def get_world_group() -> GroupCoordinator:
    return get_parallel_state().world


def get_ep_group() -> GroupCoordinator:
    return get_parallel_state().ep


def get_dp_group() -> GroupCoordinator:
    return get_parallel_state().dp


def tp_barrier(timeout_s: float | None = None) -> None:
    get_parallel_state().tp.barrier(timeout_s)


def world_barrier(timeout_s: float | None = None) -> None:
    get_parallel_state().world.barrier(timeout_s)


def destroy_parallel_state() -> None:
    """Release every group (``destroy_neuron_parallel_state``, ``neuron_parallel_state.py:1196``)."""
    global _STATE
    if _STATE is not None:
        seen = set()
        for g in _STATE.__dict__.values():
            if isinstance(g, GroupCoordinator) and g.communicator is not None and id(g.communicator) not in seen:
                seen.add(id(g.communicator))
                try:
                    g.communicator.close()
                except Exception:  # pragma: no cover
                    pass
            if isinstance(g, GroupCoordinator) and g.reducer is not None and id(g.reducer) not in seen:
                seen.add(id(g.reducer))
                g.reducer.close()
            if isinstance(g, GroupCoordinator) and g.sp_comm is not None and id(g.sp_comm) not in seen:
                seen.add(id(g.sp_comm))
                g.sp_comm.close()
    _STATE = None
    _ALL_PGS.clear()
