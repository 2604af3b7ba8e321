"""Host-side logic of the sequence-parallel NVLink boundary, without a GPU: the receive-area
addresses a scatter GEMM gets, the slot alternation of consecutive calls, and how a layer
boundary (plain partial or an MoE layer's per-route rows) reaches the communicator with this
rank's residual rows."""

import torch

from vllm_neuron_b200.parallel.communicator import SpCommunicator
from vllm_neuron_b200.parallel.state import GroupCoordinator, RoutePartial


def _fake_sp(rank=1, world=2, max_tokens=64, hidden=32):
    sc = object.__new__(SpCommunicator)
    sc.rank, sc.world, sc.hidden, sc.num_blocks = rank, world, hidden, 8
    sc.area_bytes = -(-max_tokens * hidden * 2 // 256) * 256
    sc.slot_bytes = 2 * (sc.area_bytes + sc.GUARD_BYTES)
    sc.bases = [1 << 40, 2 << 40][:world]
    sc.local = sc.bases[rank]
    sc.calls = 0
    return sc


def test_scatter_targets_point_at_this_source_in_every_owner_and_alternate_slots():
    sc = _fake_sp()
    T, H = 16, 32
    t0 = sc.scatter_targets(T, H)
    # rank 1's rows go to source area 1 of every owner: base + header + (T / world) rows of H bf16
    assert t0 == [b + sc.HEADER_BYTES + 1 * (T // 2) * H * 2 for b in sc.bases]
    sc.calls += 1  # what boundary() does after the call that consumed t0
    t1 = sc.scatter_targets(T, H)
    assert [b - a for a, b in zip(t0, t1)] == [sc.slot_bytes] * 2


def test_can_checks_divisibility_and_capacity():
    sc = _fake_sp(max_tokens=64, hidden=32)
    assert sc.can(64, 32) and sc.can(2, 32)
    assert not sc.can(63, 32)          # rows must split evenly across the ranks
    assert not sc.can(128, 32)         # beyond the receive area
    assert not sc.can(0, 32)


class _RecordingSp:
    def __init__(self):
        self.calls = []

    def can(self, T, H):
        return T % 2 == 0

    def boundary(self, x, T, residual, w, eps, bias=None, routes=None):
        self.calls.append((x, T, residual, routes))
        return torch.full((T, residual.shape[1]), 7.0)


def test_moe_route_partial_goes_to_the_sp_kernel_with_this_ranks_residual_rows():
    g = GroupCoordinator(name="tp", ranks=[0, 1], rank=1)
    g.sp_comm = _RecordingSp()
    g.sp_active = True
    T, H, k = 6, 8, 2
    ids = torch.zeros(T, k, dtype=torch.int32)
    y = torch.randn(T * k, H)
    residual = torch.arange(T * H, dtype=torch.float32).reshape(T, H)
    out, res = g.all_reduce_add_rmsnorm(RoutePartial(y, ids, 4, 4), residual, torch.ones(H), 1e-5)
    (x, T_seen, r_seen, routes), = g.sp_comm.calls
    assert x is y and T_seen == T and routes == (ids, 4, 4)
    # the replicated residual of the first boundary becomes this rank's rows T/2 .. T
    assert torch.equal(res, residual[3:]) and r_seen is res
    assert out.shape == (T, H)
