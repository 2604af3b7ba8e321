"""Expert-parallel token all-to-all: dispatch tokens to the ranks that own their experts,
run the experts on the received rows, combine the results back.

Counterpart of the reference's ``NeuronAll2AllManager`` (``vllm_neuron/parallel/all2all.py:
56`` dispatch: build metadata, permute tokens, ``all_to_all_v``; ``:186`` combine:
``all_to_all_v`` then ``topk_reduce``), selected like it by ``all2all_backend`` (the
reference registers a "neuron" backend, ``vllm/platform.py:758``).

Semantics shared by both implementations here:
* expert e lives on EP rank ``e // E_local`` (contiguous placement); the EP group is the
  world group (EP = TP x DP);
* a rank dispatches the tokens of its slice ``[t_begin, t_end)``: all of its tokens with
  attention DP (TP = 1), a 1/TP share when tokens are replicated over TP;
* a token is sent once to every rank that owns at least one of its top-k experts, with all
  k ids and weights; the receiver's expert kernel skips the ids it does not own (and -1
  ids of unused rows);
* received rows are laid out ``[world * T]``, rank s's rows at ``s * T`` in the sender's
  token order;
* combine returns ``out [T, H]`` with the sum over ranks for the slice's tokens and zeros
  elsewhere, so under TP it is a partial sum that the layer-boundary all-reduce completes.

``FusedEpAll2All`` does this with the push kernels of ``csrc/ep_a2a.cu`` over NVLink peer
memory (no host round trip, CUDA-graph safe).  ``EpAll2All`` is the collective baseline: a
dense equal-split ``all_to_all`` of the same padded layout (NCCL on GPU, gloo on CPU).  In a
multi-node job it exchanges in two hops (``hierarchical_all_to_all``): first within each node,
to the local rank at the destination's local position, then between those positional peers
across nodes, so every row crosses the inter-node network once and the many small per-rank
messages become one message per node pair and local position (the reference's inter-node
positional peer groups, ``parallel/neuron_parallel_state.py:280``).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..logging_config import init_logger

logger = init_logger(__name__)

A2A_BACKENDS = ("allgather_reducescatter", "naive", "neuron", "b200")


def ep_slice(T: int, tp_rank: int, tp_size: int) -> tuple[int, int]:
    """Token slice a TP rank dispatches (ceil split; trailing ranks may get fewer)."""
    chunk = -(-T // tp_size)
    t0 = min(T, tp_rank * chunk)
    return t0, min(T, t0 + chunk)


def compact(ids: torch.Tensor, E_local: int, world: int, t0: int, t1: int) -> torch.Tensor:
    """send_idx [T, world]: position of token t among the tokens sent to rank d, or -1."""
    T = ids.shape[0]
    owner = torch.where(ids >= 0, ids // E_local, torch.full_like(ids, -1))
    hit = (owner.unsqueeze(-1) == torch.arange(world, device=ids.device)).any(1)  # [T, world]
    inside = torch.zeros(T, dtype=torch.bool, device=ids.device)
    inside[t0:t1] = True
    hit &= inside.unsqueeze(-1)
    pos = torch.cumsum(hit.to(torch.int32), 0) - 1
    return torch.where(hit, pos, torch.full_like(pos, -1)).to(torch.int32)


def hierarchical_all_to_all(t: torch.Tensor, node_group, peer_group) -> torch.Tensor:
    """Equal-split all-to-all of ``t`` [W, ...] (row d goes to rank d; ranks node-major,
    ``W = nodes x P``) in two hops; the result equals the flat exchange: row s holds what
    rank s sent here.  Hop 1 (``node_group``, P ranks): rows for (any node, local l) go to
    local rank l.  Hop 2 (``peer_group``, one rank per node at the same local position):
    rows for node n go to that node's peer."""
    P, N = node_group.world_size, peer_group.world_size
    W = t.shape[0]
    if W != N * P:
        raise ValueError(f"{W} rows for {N} nodes x {P} ranks")
    rest = tuple(t.shape[1:])
    # [dest node, dest local, ...] -> [dest local, dest node, ...]: one chunk per local peer
    send1 = t.reshape((N, P) + rest).transpose(0, 1).contiguous()
    if P == 1:  # one rank per node: nothing to exchange inside the node (its group is this rank)
        recv1 = send1
    else:
        recv1 = torch.empty_like(send1)  # [src local, dest node, ...]
        dist.all_to_all_single(recv1, send1, group=node_group.device_group)
    send2 = recv1.transpose(0, 1).contiguous()  # [dest node, src local, ...]
    if N == 1:  # a single node: the first hop already delivered everything
        return send2.reshape((W,) + rest)
    recv2 = torch.empty_like(send2)  # [src node, src local, ...]
    dist.all_to_all_single(recv2, send2, group=peer_group.device_group)
    return recv2.reshape((W,) + rest)


class EpAll2All:
    """Collective baseline: every rank sends T padded rows to every rank."""

    fused = False

    def __init__(self, group, hidden: int, top_k: int, hierarchy: tuple | None = None):
        self.group = group
        self.world = group.world_size
        self.rank = group.rank_in_group
        self.H, self.k = hidden, top_k
        self.hierarchy = hierarchy  # (node group, positional peer group) of a multi-node job
        self._send_idx: torch.Tensor | None = None

    def can(self, T: int) -> bool:
        return True

    def _a2a(self, t: torch.Tensor) -> torch.Tensor:
        if self.hierarchy is not None:
            return hierarchical_all_to_all(t, *self.hierarchy)
        out = torch.empty_like(t)
        dist.all_to_all_single(out, t.contiguous(), group=self.group.device_group)
        return out

    def dispatch(self, x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, E_local: int, t0: int, t1: int):
        # no host synchronisation (CUDA-graph safe): every (token, rank) pair is scattered,
        # pairs that send nothing land in a dummy row T that is dropped
        T, W, k = x.shape[0], self.world, ids.shape[1]
        send_idx = compact(ids, E_local, W, t0, t1)
        self._send_idx = send_idx
        row = torch.where(send_idx >= 0, send_idx, torch.full_like(send_idx, T)).long()  # [T, W]
        flat = (torch.arange(W, device=x.device) * (T + 1)).unsqueeze(0) + row  # [T, W]
        flat = flat.reshape(-1)
        sx = torch.zeros(W * (T + 1), x.shape[1], dtype=x.dtype, device=x.device)
        sid = torch.full((W * (T + 1), k), -1, dtype=torch.int32, device=x.device)
        sw = torch.zeros(W * (T + 1), k, dtype=torch.float32, device=x.device)
        sx.index_copy_(0, flat, x.unsqueeze(1).expand(T, W, x.shape[1]).reshape(T * W, -1))
        sid.index_copy_(0, flat, ids.to(torch.int32).unsqueeze(1).expand(T, W, k).reshape(T * W, k))
        sw.index_copy_(0, flat, w.float().unsqueeze(1).expand(T, W, k).reshape(T * W, k))
        # drop the dummy rows; rows no token was sent to keep their -1 ids
        sx, sid, sw = (t.view(W, T + 1, -1)[:, :T] for t in (sx, sid, sw))
        rx, rid, rw = self._a2a(sx), self._a2a(sid), self._a2a(sw)
        return rx.view(W * T, -1), rid.view(W * T, -1), rw.view(W * T, -1)

    def combine(self, y_recv: torch.Tensor, T: int) -> torch.Tensor:
        W = self.world
        back = self._a2a(y_recv.view(W, T, -1))  # back[d, i]: rank d's output for my row i to d
        send_idx = self._send_idx
        valid = send_idx >= 0  # [T, W]
        d_idx = torch.arange(W, device=back.device).unsqueeze(0).expand(T, W)
        rows = back[d_idx, send_idx.clamp(min=0).long()].float()  # [T, W, H]
        return (rows * valid.unsqueeze(-1)).sum(1).to(y_recv.dtype)


class FusedEpAll2All:
    """NVLink push dispatch / combine (``csrc/ep_a2a.cu``) for up to ``max_tokens`` tokens
    per rank per call; larger calls (long prefill chunks) use the collective baseline."""

    fused = True

    def __init__(self, group, device: torch.device, hidden: int, top_k: int, max_tokens: int = 256):
        from ..ops import _ext, device_status

        _ext.load()
        self.group = group
        self.device = device
        self.world = group.world_size
        self.rank = group.rank_in_group
        self.H, self.k = hidden, top_k
        self.Tc = max(4, min(256, (max_tokens + 3) // 4 * 4))
        self.cpd = max(1, min(16, 128 // self.world))
        sb = self.world * self.Tc * (4 * hidden + 8 * top_k)
        self.slot_bytes = (sb + 255) // 256 * 256
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
        W, Tc = self.world, self.Tc
        self.x_recv = torch.empty(W * Tc, hidden, dtype=torch.bfloat16, device=device)
        self.ids_recv = torch.empty(W * Tc, top_k, dtype=torch.int32, device=device)
        self.w_recv = torch.empty(W * Tc, top_k, dtype=torch.float32, device=device)
        self.send_idx = torch.empty(Tc, W, dtype=torch.int32, device=device)
        self.status = device_status(device)
        self.fallback = EpAll2All(group, hidden, top_k)
        self._last_fused = True
        group.barrier()
        logger.info("fused EP all-to-all: %d ranks, %d tokens per call, %.1f MB per rank", W, Tc,
                    (2 * self.slot_bytes) / 1e6)

    def can(self, T: int) -> bool:
        return T <= self.Tc

    def dispatch(self, x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, E_local: int, t0: int, t1: int):
        T = x.shape[0]
        self._last_fused = self.can(T) and x.dtype == torch.bfloat16
        if not self._last_fused:
            return self.fallback.dispatch(x, ids, w, E_local, t0, t1)
        W = self.world
        xr, ir, wr = self.x_recv[:W * T], self.ids_recv[:W * T], self.w_recv[:W * T]
        torch.ops.b200.ep_dispatch(self.bases, self.rank, self.slot_bytes, self.cpd, self.Tc, E_local, t0, t1,
                                   x.contiguous(), ids.to(torch.int32).contiguous(), w.float().contiguous(), xr, ir,
                                   wr, self.send_idx, self.status)
        return xr, ir, wr

    def combine(self, y_recv: torch.Tensor, T: int) -> torch.Tensor:
        if not self._last_fused:
            return self.fallback.combine(y_recv, T)
        out = torch.empty(T, self.H, dtype=torch.bfloat16, device=y_recv.device)
        torch.ops.b200.ep_combine(self.bases, self.rank, self.slot_bytes, self.cpd, self.Tc,
                                  y_recv.contiguous(), self.ids_recv[:self.world * T], self.send_idx, out, self.status)
        return out

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


def make_ep_all2all(backend: str, group, device: torch.device, hidden: int, top_k: int, max_tokens: int = 256,
                    ps=None):
    """The all-to-all object for ``all2all_backend`` (None: all-gather / reduce-scatter path).
    Collective when it builds the fused path: every rank of ``group`` calls it.  ``ps``: the
    parallel state; in a multi-node job whose EP group is the whole world the collective path
    exchanges hierarchically."""
    if backend not in A2A_BACKENDS:
        raise ValueError(f"all2all_backend must be one of {A2A_BACKENDS}, got {backend!r}")
    if backend == "allgather_reducescatter" or group.world_size == 1:
        return None
    multi_node = ps is not None and getattr(ps, "nnodes", 1) > 1 and ps.node is not None
    if backend in ("neuron", "b200") and device.type == "cuda" and group.world_size <= 8 and not multi_node:
        return FusedEpAll2All(group, device, hidden, top_k, max_tokens)
    hier = None
    if multi_node and list(group.ranks) == list(range(ps.world.world_size)):
        hier = (ps.node, ps.inter_node)
    return EpAll2All(group, hidden, top_k, hier)
