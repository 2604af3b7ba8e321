"""Collective microbenchmarks (one process per GPU, under torchrun).

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m vllm_neuron_b200.benchmarks.collectives
    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m vllm_neuron_b200.benchmarks.collectives --op ep

``--op ep`` times the EP all-to-all (see ``_ep``); ``--op gemm_ar`` the row-parallel GEMM
fused with the all-reduce (see ``_gemm_ar``); ``--op sp --tokens 512,2048,4096`` the
sequence-parallel prefill boundary (see ``_sp``); the default is the layer-boundary all-reduce:

For each token count T (hidden 2880, bf16) it times, with CUDA events after warm-up and as
the maximum over ranks:
* ``fused``: the one-shot NVLink all-reduce fused with bias + residual add + RMSNorm
  (``csrc/comm.cu``), inside a CUDA graph of ``--iters`` back-to-back calls;
* ``nccl``: NCCL all-reduce followed by the fused add + RMSNorm kernel, same graph setup.

Roofline of the fused path: every rank must read the other ranks' partial rows over NVLink,
(world - 1) * T * H * 2 bytes, at the measured 770 GB/s per direction, so
``target_us = bytes / 770e3``; ``frac`` = target / achieved.  One JSON line per (T, path) on
rank 0.
"""

from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

LINK_GBS = 770.0


def _ep(a, rank, world, dev, ps) -> None:
    """EP all-to-all: fused NVLink dispatch + combine (identity experts) in a CUDA graph of
    ``--iters`` calls, and the collective (NCCL) all-to-all baseline timed eagerly.  Roofline:
    the rows that must leave this rank (each token once to every other rank owning one of its
    top-k experts, H bf16 + k ids / weights) and come back (H bf16), over 770 GB/s."""
    from vllm_neuron_b200.parallel.all2all import EpAll2All, FusedEpAll2All

    H, k, E = a.hidden, 4, a.experts
    E_local = E // world
    fused = FusedEpAll2All(ps.world, dev, H, k, max_tokens=256)
    coll = EpAll2All(ps.world, H, k)
    for T in [int(t) for t in a.tokens.split(",")]:
        torch.manual_seed(1000 + rank)
        x = torch.randn(T, H, device=dev).bfloat16()
        ids = torch.stack([torch.randperm(E, device=dev)[:k] for _ in range(T)]).to(torch.int32)
        w = torch.rand(T, k, device=dev)
        owners = (ids // E_local).long()
        remote = sum(int(((owners == d).any(1)).sum()) for d in range(world) if d != rank)
        nbytes = remote * (H * 2 + 8 * k) + remote * H * 2
        t_max = torch.tensor([float(nbytes)], device=dev)
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
        nbytes = int(t_max.item())
        res = {}
        for path, a2a in (("fused", fused), ("nccl", coll)):
            def step():
                xr, ir, wr = a2a.dispatch(x, ids, w, E_local, 0, T)
                return a2a.combine(xr, T)

            for _ in range(3):
                step()
            torch.cuda.synchronize()
            if path == "fused":
                g = torch.cuda.CUDAGraph()
                s = torch.cuda.Stream()
                s.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(s):
                    step()
                torch.cuda.current_stream().wait_stream(s)
                with torch.cuda.graph(g):
                    for _ in range(a.iters):
                        step()
                g.replay()
                run = g.replay
                n = a.iters
            else:
                run = step
                n = 1
            dist.barrier()
            torch.cuda.synchronize()
            times = []
            for _ in range(5 if path == "fused" else a.iters):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                run()
                e1.record()
                torch.cuda.synchronize()
                times.append(e0.elapsed_time(e1) * 1000.0 / n)
            t = torch.tensor([sum(times) / len(times)], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            res[path] = t.item()
            if path == "fused":
                del g
        target = nbytes / (LINK_GBS * 1e3)
        if rank == 0:
            for path, us in res.items():
                print(json.dumps({"op": "ep_dispatch_combine", "path": path, "world": world, "T": T, "H": H,
                                  "E": E, "k": k, "us": round(us, 2), "nvlink_bytes_per_rank": nbytes,
                                  "target_us": round(target, 2), "frac_of_roofline": round(target / us, 3)}),
                      flush=True)
    fused.close()


def _gemm_ar(a, rank, world, dev, ps) -> None:
    """Row-parallel projection + layer boundary (GPT-OSS o_proj: [T, 4096 / world] x
    [2880, 4096 / world]^T, then all-reduce + bias + residual + RMSNorm), CUDA graph of
    ``--iters`` calls, max over ranks:
    * ``nvls``: the tcgen05 GEMM adds its fp32 output tiles into every rank's accumulator
      with multimem reductions (NVSwitch), one finish kernel normalises;
    * ``gemm+fused_ar``: the same GEMM storing bf16, then the one-shot NVLink all-reduce
      kernel fused with the norm;
    * ``cublas+nccl``: library GEMM, NCCL all-reduce, add + RMSNorm kernel (baseline).
    Roofline: the slower of the weight stream at the measured HBM bandwidth, the GEMM at the
    measured bf16 peak and the bytes each rank must push (fp32 rows once through the switch
    for nvls, bf16 rows to every peer otherwise) at 770 GB/s."""
    import torch.nn.functional as F

    from vllm_neuron_b200 import ops

    tp = ps.tp
    H, Kr = a.hidden, 4096 // world
    hbm, peak = 6537.0, 1667.1
    try:
        with open(os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")) as f:
            mp_ = json.load(f)
            hbm, peak = float(mp_["hbm_gbs"]), float(mp_["bf16_tflops"])
    except (OSError, ValueError, KeyError):
        pass
    nw = torch.ones(H, device=dev)
    torch.manual_seed(7 + rank)
    W = (torch.randn(H, Kr, device=dev) * 0.02).bfloat16()
    for T in [int(t) for t in a.tokens.split(",")]:
        x = torch.randn(T, Kr, device=dev).bfloat16()
        res = torch.randn(T, H, device=dev).bfloat16()
        bias = torch.zeros(H, device=dev).bfloat16()
        paths = (["nvls"] if tp.reducer is not None else []) + ["gemm+fused_ar", "cublas+nccl"]
        for path in paths:
            def step():
                if path == "nvls":
                    return tp.reducer.linear_add_rmsnorm(x, W, res, nw, 1e-5, bias)
                if path == "gemm+fused_ar":
                    return tp.communicator.all_reduce_add_rmsnorm(ops.linear(x, W), res, nw, 1e-5, bias)
                y = F.linear(x, W)
                dist.all_reduce(y, group=tp.device_group)
                return ops.fused_add_rms_norm(y + bias, res, nw, 1e-5)

            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                for _ in range(3):
                    step()
            torch.cuda.current_stream().wait_stream(s)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for _ in range(a.iters):
                    step()
            for _ in range(3):
                g.replay()
            dist.barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            g.replay()
            e1.record()
            torch.cuda.synchronize()
            t = torch.tensor([e0.elapsed_time(e1) * 1000.0 / a.iters], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            us = t.item()
            link_bytes = T * H * 4 if path == "nvls" else (world - 1) * T * H * 2
            t_link = link_bytes / (LINK_GBS * 1e3)
            t_hbm = H * Kr * 2 / (hbm * 1e3)
            t_mma = 2.0 * T * H * Kr / (peak * 1e6)
            target = max(t_link, t_hbm, t_mma)
            if rank == 0:
                print(json.dumps({"op": "gemm_allreduce_rmsnorm", "path": path, "world": world, "T": T, "H": H,
                                  "K_per_rank": Kr, "us": round(us, 2), "target_us": round(target, 2),
                                  "bound": ["nvlink", "hbm", "mma"][[t_link, t_hbm, t_mma].index(target)],
                                  "frac_of_roofline": round(target / us, 3)}), flush=True)
            del g


def _sp(a, rank, world, dev, ps) -> None:
    """Sequence-parallel prefill boundary after the row-parallel o_proj (GPT-OSS: [T, 4096 /
    world] x [2880, 4096 / world]^T, then reduce-scatter + bias + residual + RMSNorm +
    all-gather), CUDA graph of ``--iters`` calls, max over ranks:
    * ``gemm_scatter+sp``: the tcgen05 GEMM stores each partial row block straight into its
      owner's receive area (peer stores from the epilogue), then the boundary kernel reduces,
      normalises and pushes the rows to every rank;
    * ``gemm+sp``: the GEMM into local memory, then the boundary kernel with both push phases;
    * ``cublas+nccl``: library GEMM, NCCL reduce-scatter, bias add, add + RMSNorm kernel, NCCL
      all-gather (baseline);
    * ``sp`` / ``nccl``: the collective part alone on a precomputed partial.
    Roofline: every rank must send (world - 1) / world of the T x H bf16 partial (the
    reduce-scatter) and of the normalised rows (the all-gather) over NVLink at 770 GB/s; with
    the GEMM, the slower of that, the weight stream at HBM bandwidth and the MMA at the bf16 peak."""
    import torch.nn.functional as F

    from vllm_neuron_b200 import ops
    from vllm_neuron_b200.parallel.communicator import attach_sp_communicator

    tp = ps.tp
    H, Kr = a.hidden, 4096 // world
    toks = [int(t) for t in a.tokens.split(",")]
    attach_sp_communicator(ps, dev, max(toks), H)
    sc = tp.sp_comm
    hbm, peak = 6537.0, 1667.1
    try:
        with open(os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")) as f:
            mp_ = json.load(f)
            hbm, peak = float(mp_["hbm_gbs"]), float(mp_["bf16_tflops"])
    except (OSError, ValueError, KeyError):
        pass
    nw = torch.ones(H, device=dev)
    torch.manual_seed(7 + rank)
    W = (torch.randn(H, Kr, device=dev) * 0.02).bfloat16()
    for T in toks:
        Ts = T // world
        x = torch.randn(T, Kr, device=dev).bfloat16()
        part = ops.linear(x, W)
        res = torch.randn(Ts, H, device=dev).bfloat16()
        bias = torch.zeros(H, device=dev).bfloat16()
        for path in ("gemm_scatter+sp", "gemm+sp", "cublas+nccl", "sp", "nccl"):
            def step():
                if path == "gemm_scatter+sp":
                    ops.linear_scatter(x, W, sc.scatter_targets(T, H), H)
                    return sc.boundary(None, T, res, nw, 1e-5, bias)
                if path in ("gemm+sp", "sp"):
                    return sc.boundary(ops.linear(x, W) if path == "gemm+sp" else part, T, res, nw, 1e-5, bias)
                y = F.linear(x, W) if path == "cublas+nccl" else part
                ys = torch.empty(Ts, H, device=dev, dtype=y.dtype)
                dist.reduce_scatter_tensor(ys, y, group=tp.device_group)
                o, _ = ops.fused_add_rms_norm(ys + bias, res, nw, 1e-5)
                full = torch.empty(T, H, device=dev, dtype=o.dtype)
                dist.all_gather_into_tensor(full, o, group=tp.device_group)
                return full

            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                for _ in range(3):
                    step()
            torch.cuda.current_stream().wait_stream(s)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for _ in range(a.iters):
                    step()
            for _ in range(3):
                g.replay()
            dist.barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            g.replay()
            e1.record()
            torch.cuda.synchronize()
            t = torch.tensor([e0.elapsed_time(e1) * 1000.0 / a.iters], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            us = t.item()
            link_bytes = 2 * (world - 1) * Ts * H * 2
            t_link = link_bytes / (LINK_GBS * 1e3)
            gemm = path not in ("sp", "nccl")
            t_hbm = H * Kr * 2 / (hbm * 1e3) if gemm else 0.0
            t_mma = 2.0 * T * H * Kr / (peak * 1e6) if gemm else 0.0
            target = max(t_link, t_hbm, t_mma)
            if rank == 0:
                print(json.dumps({"op": "sp_boundary", "path": path, "world": world, "T": T, "H": H,
                                  "K_per_rank": Kr, "us": round(us, 2), "nvlink_bytes_per_rank": link_bytes,
                                  "target_us": round(target, 2),
                                  "bound": ["nvlink", "hbm", "mma"][[t_link, t_hbm, t_mma].index(target)],
                                  "frac_of_roofline": round(target / us, 3)}), flush=True)
            del g
    ok = sc.check_canaries()
    if rank == 0:
        print(json.dumps({"op": "sp_boundary", "guards_intact": ok}), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", choices=["allreduce", "ep", "gemm_ar", "sp"], default="allreduce")
    ap.add_argument("--hidden", type=int, default=2880)
    ap.add_argument("--tokens", default="1,16,64,256")
    ap.add_argument("--experts", type=int, default=128)
    ap.add_argument("--iters", type=int, default=50)
    a = ap.parse_args()
    from vllm_neuron_b200 import ops
    from vllm_neuron_b200.parallel import state as pstate
    from vllm_neuron_b200.parallel.communicator import attach_communicators, attach_reducers

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pstate.init_distributed_environment(world, rank, backend="nccl", local_rank=local, timeout_s=120)
    ps = pstate.initialize_parallel_state(tp=world, timeout_s=120)
    if a.op == "ep":
        _ep(a, rank, world, dev, ps)
        torch.cuda.synchronize()
        pstate.destroy_parallel_state()
        dist.destroy_process_group()
        return
    if a.op == "sp":
        _sp(a, rank, world, dev, ps)
        torch.cuda.synchronize()
        pstate.destroy_parallel_state()
        dist.destroy_process_group()
        return
    attach_communicators(ps, dev)
    if a.op == "gemm_ar":
        attach_reducers(ps, dev)
        _gemm_ar(a, rank, world, dev, ps)
        torch.cuda.synchronize()
        pstate.destroy_parallel_state()
        dist.destroy_process_group()
        return
    tp = ps.tp
    H = a.hidden
    w = torch.ones(H, device=dev)
    for T in [int(t) for t in a.tokens.split(",")]:
        x = torch.randn(T, H, device=dev).bfloat16()
        res = torch.randn(T, H, device=dev).bfloat16()
        bias = torch.zeros(H, device=dev).bfloat16()
        for path in ("fused", "nccl"):
            comm = tp.communicator

            def step():
                if path == "fused":
                    return comm.all_reduce_add_rmsnorm(x, res, w, 1e-5, bias)
                y = tp.all_reduce(x.clone()) if comm is None else _nccl(tp, x)
                return ops.fused_add_rms_norm(y + bias, res, w, 1e-5)

            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                for _ in range(3):
                    step()
            torch.cuda.current_stream().wait_stream(s)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for _ in range(a.iters):
                    step()
            for _ in range(3):
                g.replay()
            dist.barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            g.replay()
            e1.record()
            torch.cuda.synchronize()
            t = torch.tensor([e0.elapsed_time(e1) * 1000.0 / a.iters], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            us = t.item()
            nbytes = (world - 1) * T * H * 2
            target = nbytes / (LINK_GBS * 1e3)
            if rank == 0:
                print(json.dumps({"path": path, "world": world, "T": T, "H": H, "us": round(us, 2),
                                  "nvlink_bytes_per_rank": nbytes, "target_us": round(target, 2),
                                  "frac_of_roofline": round(target / us, 3)}), flush=True)
            del g
    torch.cuda.synchronize()
    pstate.destroy_parallel_state()
    dist.destroy_process_group()


def _nccl(tp, x):
    y = x.clone()
    dist.all_reduce(y, group=tp.device_group)
    return y


if __name__ == "__main__":
    main()
