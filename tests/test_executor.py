"""MPExecutor (multi-process test harness) on CPU gloo ranks, including host-side failure
detection: a rank that raises, a rank that exits, a rank that stops answering."""

import os
import time

import pytest
import torch


def _allreduce(ctx, base):
    t = torch.tensor([float(base + ctx.rank)])
    return ctx.ps.tp.all_reduce(t).item()


def _make(ctx, scale):
    return {"w": scale * (ctx.rank + 1)}


def _use(ctx):
    return ctx.obj["w"]


def _layout(ctx):
    return (ctx.ps.tp.world_size, ctx.ps.dp.world_size)


def _raise_on_1(ctx):
    if ctx.rank == 1:
        raise ValueError("injected failure")
    return ctx.rank


def _exit_on_1(ctx):
    if ctx.rank == 1:
        os._exit(3)
    return ctx.rank


def _stall_on_0(ctx):
    if ctx.rank == 0:
        time.sleep(30)
    return ctx.rank


def test_executor_run_load_reinit():
    from vllm_neuron_b200.utils.executor import MPExecutor

    with MPExecutor(world_size=2, tp=2, timeout_s=60) as ex:
        assert ex.run(_allreduce, 10) == [21.0, 21.0]
        ex.load(_make, 3)
        assert ex.run(_use) == [3, 6]
        assert ex.run(_layout) == [(2, 1), (2, 1)]
        ex.reinit(tp=1, dp=2)
        assert ex.run(_layout) == [(1, 2), (1, 2)]


def test_executor_reports_rank_exception():
    from vllm_neuron_b200.utils.executor import MPExecutor, RankError

    with MPExecutor(world_size=2, tp=2, timeout_s=60) as ex:
        with pytest.raises(RankError) as ei:
            ex.run(_raise_on_1)
        assert ei.value.rank == 1 and "injected failure" in str(ei.value)
        assert ex.run(_layout) == [(2, 1), (2, 1)]  # the pool survives a task error


def test_executor_detects_dead_and_stalled_ranks():
    from vllm_neuron_b200.utils.executor import MPExecutor, RankError

    ex = MPExecutor(world_size=2, tp=2, timeout_s=60)
    with pytest.raises(RankError) as ei:
        ex.run(_exit_on_1)
    assert ei.value.rank == 1 and "exited" in str(ei.value)
    ex = MPExecutor(world_size=2, tp=2, timeout_s=4)
    t0 = time.monotonic()
    with pytest.raises(RankError) as ei:
        ex.run(_stall_on_0)
    assert ei.value.rank == 0 and time.monotonic() - t0 < 20


def _ep_a2a_case(ctx, T, t0, t1):
    from vllm_neuron_b200.parallel.all2all import EpAll2All

    W, H, k, E = ctx.ps.world.world_size, 16, 2, 8
    E_local = E // W
    g = torch.Generator().manual_seed(10 + ctx.rank)
    x = torch.randn(T, H, generator=g)
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32)
    w = torch.rand(T, k, generator=g)
    a2a = EpAll2All(ctx.ps.world, H, k)
    xr, ir, wr = a2a.dispatch(x, ids, w, E_local, t0, t1)
    off = ctx.rank * E_local
    local = (ir >= off) & (ir < off + E_local)
    yr = xr * torch.where(local, wr * (ir.float() + 1), torch.zeros_like(wr)).sum(-1, keepdim=True)
    out = a2a.combine(yr, T)
    want = x * (w * (ids.float() + 1)).sum(-1, keepdim=True)
    want[:t0] = 0
    want[t1:] = 0
    return (out - want).abs().max().item()


def test_collective_all2all_matches_math():
    """The collective EP all-to-all (gloo): dispatch to expert owners, per-rank experts,
    combine; whole batch and a TP-style slice."""
    from vllm_neuron_b200.utils.executor import MPExecutor

    with MPExecutor(world_size=2, tp=2, timeout_s=120) as ex:
        assert max(ex.run(_ep_a2a_case, 9, 0, 9)) < 1e-5
        assert max(ex.run(_ep_a2a_case, 9, 2, 6)) < 1e-5


def _lockstep(ctx, skew_rank, skew, tag_rank):
    """Every rank reduces once; ``skew_rank`` claims a later step, ``tag_rank`` another call site."""
    step = 7 + (skew if ctx.rank == skew_rank else 0)
    tag = 2 if ctx.rank == tag_rank else 1
    try:
        return ("ok", ctx.ps.world.lockstep_all_reduce_max([ctx.rank * 10, 5], step, tag))
    except RuntimeError as e:
        return ("tripped", str(e))


def test_dp_lockstep_tripwire_fires_on_every_rank():
    """A replica one step ahead, or at a different reduce, makes every rank raise; aligned
    ranks get the plain MAX-reduce."""
    from vllm_neuron_b200.utils.executor import MPExecutor

    with MPExecutor(world_size=2, tp=1, dp=2, timeout_s=60) as ex:
        assert ex.run(_lockstep, -1, 0, -1) == [("ok", [10, 5]), ("ok", [10, 5])]
        res = ex.run(_lockstep, 1, 1, -1)  # rank 1 skipped a step
        assert [r[0] for r in res] == ["tripped", "tripped"] and "steps 7..8" in res[0][1]
        res = ex.run(_lockstep, -1, 0, 0)  # rank 0 at the token-count reduce, rank 1 at the flags reduce
        assert [r[0] for r in res] == ["tripped", "tripped"] and "call sites 1..2" in res[1][1]


def _shard_sum(ctx, shard):
    return float(shard.sum()) + 1000 * ctx.rank


def _where(ctx):
    return (ctx.nnodes, ctx.node_rank, ctx.local_rank)


def _matmul(ctx, n):
    a = torch.randn(n, n)
    return float((a @ a).sum() * 0)


def test_executor_per_rank_inputs_nodes_profile_and_pool(tmp_path):
    """Per-rank arguments, simulated nodes, per-rank Chrome traces, and the pooled executor
    that a second request with another layout reuses (re-laid-out, same processes)."""
    from vllm_neuron_b200.utils.executor import MPExecutor

    with MPExecutor(world_size=4, tp=2, dp=2, nnodes=2, timeout_s=60) as ex:
        x = torch.arange(8.0)
        assert ex.run_per_rank(_shard_sum, [(c,) for c in x.chunk(4)]) == [1.0, 1005.0, 2009.0, 3013.0]
        assert ex.run(_where) == [(2, 0, 0), (2, 0, 1), (2, 1, 0), (2, 1, 1)]
        ex.start_profile(str(tmp_path / "prof"))
        ex.run(_matmul, 64)
        paths = ex.stop_profile()
        assert [os.path.basename(p) for p in paths] == [f"trace_rank{r}.json" for r in range(4)]
        assert all(os.path.getsize(p) > 0 for p in paths)
        with pytest.raises(ValueError):
            ex.run_per_rank(_shard_sum, [(x,)])
    try:
        a = MPExecutor.shared(2, tp=2)
        pids = [p.pid for p in a._procs]
        b = MPExecutor.shared(2, tp=1, dp=2)
        assert b is a and [p.pid for p in b._procs] == pids
        assert b.run(_layout) == [(1, 2), (1, 2)]
    finally:
        MPExecutor.shutdown_shared()


def _hier_case(ctx, T, H):
    """Flat vs two-hop all-to-all of the same per-rank data, and EP dispatch + combine through
    both exchanges (experts: a fixed per-expert scale)."""
    import torch.distributed as dist

    from vllm_neuron_b200.parallel.all2all import EpAll2All, hierarchical_all_to_all

    ps = ctx.ps
    W = ps.world.world_size
    g = torch.Generator().manual_seed(100 + ctx.rank)
    t = torch.randn(W, T, H, generator=g)
    flat = torch.empty_like(t)
    dist.all_to_all_single(flat, t, group=ps.world.device_group)
    hier = hierarchical_all_to_all(t, ps.node, ps.inter_node)
    exact = bool(torch.equal(flat, hier))
    E_local, k = 2, 2
    x = torch.randn(T, H, generator=g)
    ids = torch.stack([torch.randperm(E_local * W, generator=g)[:k] for _ in range(T)])
    w = torch.rand(T, k, generator=g)
    outs = []
    for a2a in (EpAll2All(ps.world, H, k), EpAll2All(ps.world, H, k, (ps.node, ps.inter_node))):
        rx, rid, rw = a2a.dispatch(x, ids, w, E_local, 0, T)
        lo = ctx.rank * E_local
        y = torch.zeros_like(rx)
        for j in range(k):
            e = rid[:, j].long()
            mine = (e >= lo) & (e < lo + E_local)
            y += torch.where(mine[:, None], rx * (1.0 + e[:, None].float()) * rw[:, j:j + 1], torch.zeros_like(rx))
        outs.append(a2a.combine(y, T))
    want = sum(x * (1.0 + ids[:, j:j + 1].float()) * w[:, j:j + 1] for j in range(k))
    return exact, float((outs[0] - outs[1]).abs().max()), float((outs[1] - want).abs().max()), ps.degrees["nnodes"]


def test_hierarchical_all_to_all_two_nodes():
    """Two simulated nodes of two ranks: the node and positional-peer groups exist, the two-hop
    exchange equals the flat one bit for bit, and the EP all-to-all gives the same combined
    output through either."""
    from vllm_neuron_b200.parallel.state import build_node_group_ranks
    from vllm_neuron_b200.utils.executor import MPExecutor

    assert build_node_group_ranks(16, 2) == ([list(range(8)), list(range(8, 16))],
                                             [[i, i + 8] for i in range(8)])
    with MPExecutor(world_size=4, tp=4, nnodes=2, timeout_s=120) as ex:
        for exact, d_paths, d_math, nn in ex.run(_hier_case, 5, 16):
            assert exact and d_paths < 1e-6 and d_math < 1e-4 and nn == 2


def test_hierarchical_all_to_all_one_rank_per_node():
    """Two simulated nodes of one rank each: the node groups have a single rank, so the
    in-node hop is skipped and the exchange still equals the flat one."""
    from vllm_neuron_b200.utils.executor import MPExecutor

    with MPExecutor(world_size=2, tp=2, nnodes=2, timeout_s=120) as ex:
        for exact, d_paths, d_math, nn in ex.run(_hier_case, 3, 8):
            assert exact and d_paths < 1e-6 and d_math < 1e-4 and nn == 2
