"""Headline benchmark: GPT-OSS-120B (MXFP4 experts) output tokens/s at concurrency 64.

``python bench.py --gpus N --steps K --warmup W`` (N > 1 under torch.distributed.run).

Workload (BASELINE.json config 3 shape): a closed serving loop that keeps 64 requests in
flight, the way ``vllm bench serve --max-concurrency 64`` drives a server.  Every request has
2048 synthetic random prompt tokens and generates 512 tokens (greedy, ignore EOS); weights are
random-init with the GPT-OSS-120B architecture (36 layers, hidden 2880, 64 q / 8 kv heads of
64, 128 experts top-4, MXFP4 experts, bf16 rest).  When a request finishes, a new one is
submitted at once, so the engine alternates one 2048-token prefill (admission of the
replacement) with about eight decode steps at batch 64: the steady state of serving at
concurrency 64, whose output rate is the headline metric.  The 64 first requests get staggered
output lengths (8, 16, ..., 512 tokens) so that completions are evenly spread from the start.

A benchmark *step* is one serving period of that steady state: from one completion to the
next (the replacement's prefill plus the decode steps until the next request finishes).
W periods are run untimed, then K periods are timed:
* ``value``  output tokens of the K periods / device time, where device time is the sum of
  every engine step's GPU span (CUDA events recorded around each step's H2D staging, forward,
  sampling and D2H enqueue; host gaps between steps excluded), max over ranks.  The weights
  (~60 GB) and KV cache exceed L2 many times over every step, so no flush is needed.
* ``e2e``    the same output tokens / wall-clock time of the same window through the public
  engine API (``LLMEngine.add_request`` / ``LLMEngine.step``): scheduling, pinned-memory H2D
  of every step's inputs, the forward, and the D2H read of the sampled ids, max over ranks.
* ``config.ttft_p50_ms`` / ``tpot_p50_ms``: medians over the requests of the window (arrival
  to first token; per-request mean interval between later tokens).  ``decode_only_tok_s``:
  K x 8 replays of the captured batch-64 decode graph between CUDA events (no prefill).
Parallelism for N GPUs: attention TP=N (heads), experts EP=N; each layer boundary is one
fused NVLink all-reduce + residual + RMSNorm kernel; total concurrency stays 64 (strong
scaling).  ``--impl reference`` reports why the reference plugin cannot run here.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

GPT_OSS_120B = {
    "architectures": ["GptOssForCausalLM"], "model_type": "gpt_oss", "vocab_size": 201088, "hidden_size": 2880,
    "num_hidden_layers": 36, "num_attention_heads": 64, "num_key_value_heads": 8, "head_dim": 64,
    "intermediate_size": 2880, "num_local_experts": 128, "num_experts_per_tok": 4, "sliding_window": 128,
    "layer_types": ["sliding_attention" if i % 2 == 0 else "full_attention" for i in range(36)],
    "rope_theta": 150000.0,
    "rope_scaling": {"rope_type": "yarn", "factor": 32.0, "beta_fast": 32.0, "beta_slow": 1.0,
                     "original_max_position_embeddings": 4096, "truncate": False},
    "rms_norm_eps": 1e-5, "swiglu_limit": 7.0, "attention_bias": True, "max_position_embeddings": 131072,
    "quantization_config": {"quant_method": "mxfp4"}, "eos_token_id": 200002,
}
GPT_OSS_20B = dict(GPT_OSS_120B, num_hidden_layers=24, num_local_experts=32,
                   layer_types=["sliding_attention" if i % 2 == 0 else "full_attention" for i in range(24)])
METRIC = "output tok/s at fixed concurrency (GPT-OSS-120B, 8×B200); p50 TTFT / TPOT"
# Device-timed value of ``--baseline-of-record`` (this framework with cuBLAS dense layers and NCCL
# collectives) measured on a B200, per (model, GPUs); the reference publishes no number for this
# configuration.  vs_baseline = value / it.
BASELINE_OF_RECORD: dict = {("gpt-oss-120b", 1): 3325.27}


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                p = [x.strip() for x in line.split(",")]
                if len(p) >= 9:
                    rows.append(p)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows),
                "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())}


def run_reference(args) -> None:
    """The reference is a Trainium plugin: its model and functional packages import the
    Neuron SDK (``nki``) at module level and its package init hides every CUDA device."""
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    sys.path.insert(0, ref_dir)
    reason = None
    if not os.path.isdir(os.path.join(ref_dir, "vllm_neuron")):
        reason = ("the reference is not installed in baseline/_ref on this machine (pip install --no-deps "
                  "--target baseline/_ref of the reference tree); it targets AWS Trainium and cannot run on B200")
    try:
        import vllm_neuron.functional  # noqa: F401
    except Exception as e:  # noqa: BLE001
        reason = reason or (f"the reference installs (baseline/_ref) but cannot run on B200: "
                  f"importing vllm_neuron.functional fails ({type(e).__name__}: {e}); it targets AWS Trainium "
                  f"(NKI kernels, neuronx-cc) and sets CUDA_VISIBLE_DEVICES='' at import")
    rank = int(os.environ.get("RANK", "0"))
    if rank == 0:
        print(json.dumps({"impl": "reference", "unavailable": reason or "reference has no CUDA execution path"}))


def _count_our_kernels(fn) -> tuple[int, int, str]:
    """Run ``fn`` under torch.profiler (CUDA activity): (launches of this library's kernels,
    all kernel launches, per-kernel table)."""
    import torch

    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    ours = total = 0
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA:
            total += 1
            if "b200::" in ev.name:
                ours += 1
    table = prof.key_averages().table(sort_by="self_cuda_time_total", row_limit=40)
    return ours, total, table


def _collective_check(eng, H: int, T: int = 64) -> dict:
    """At N > 1, before timing: the fused layer-boundary collectives on the benchmark's shapes
    against NCCL + the plain kernels (same inputs on every rank), as max |difference| of the
    normalised output and of the new residual.  Every rank runs the same calls."""
    import torch
    import torch.distributed as dist
    import torch.nn.functional as F

    from vllm_neuron_b200 import ops

    tp = eng.worker.ps.tp
    dev = eng.worker.device
    g = torch.Generator(device=dev).manual_seed(100 + dist.get_rank())
    res = {}
    x = torch.randn(T, H, device=dev, generator=g).bfloat16()
    r0 = torch.randn(T, H, device=dev, generator=torch.Generator(device=dev).manual_seed(7)).bfloat16()
    w = torch.ones(H, device=dev)
    ref_sum = x.float().clone()
    dist.all_reduce(ref_sum, group=tp.device_group)
    want_out, want_res = ops.fused_add_rms_norm(ref_sum.bfloat16(), r0.clone(), w, 1e-5)
    if tp.communicator is not None and tp.communicator.can_all_reduce(x):
        out, rr = tp.communicator.all_reduce_add_rmsnorm(x, r0.clone(), w, 1e-5)
        res["fused_allreduce_rmsnorm_max_err"] = max((out.float() - want_out.float()).abs().max().item(),
                                                     (rr.float() - want_res.float()).abs().max().item())
    if tp.reducer is not None:
        K = 4096 // tp.world_size
        a = torch.randn(T, K, device=dev, generator=g).bfloat16()
        wt = (torch.randn(H, K, device=dev, generator=torch.Generator(device=dev).manual_seed(9)) * 0.02).bfloat16()
        y = F.linear(a, wt).float()
        dist.all_reduce(y, group=tp.device_group)
        want_out, want_res = ops.fused_add_rms_norm(y.bfloat16(), r0.clone(), w, 1e-5)
        out, rr = tp.reducer.linear_add_rmsnorm(a, wt, r0.clone(), w, 1e-5, None)
        res["nvls_gemm_allreduce_rmsnorm_max_err"] = max((out.float() - want_out.float()).abs().max().item(),
                                                         (rr.float() - want_res.float()).abs().max().item())
    sc = tp.sp_comm
    Tp = 2048
    if sc is not None and sc.can(Tp, H):
        # prefill SP boundary on the prompt's shape: the scatter GEMM + the boundary kernel
        # against cuBLAS + NCCL reduce-scatter + norm + NCCL all-gather
        K = 4096 // tp.world_size
        Ts, r = Tp // tp.world_size, tp.rank_in_group
        a = torch.randn(Tp, K, device=dev, generator=g).bfloat16()
        wt = (torch.randn(H, K, device=dev, generator=torch.Generator(device=dev).manual_seed(9)) * 0.02).bfloat16()
        rp = torch.randn(Tp, H, device=dev, generator=torch.Generator(device=dev).manual_seed(8)).bfloat16()
        y = F.linear(a, wt).float()
        dist.all_reduce(y, group=tp.device_group)
        want_out, want_res = ops.fused_add_rms_norm(y[r * Ts:(r + 1) * Ts].bfloat16(),
                                                    rp[r * Ts:(r + 1) * Ts].clone(), w, 1e-5)
        want_full = torch.empty(Tp, H, device=dev, dtype=torch.bfloat16)
        dist.all_gather_into_tensor(want_full, want_out.contiguous(), group=tp.device_group)
        rr = rp[r * Ts:(r + 1) * Ts].clone()
        ops.linear_scatter(a, wt, sc.scatter_targets(Tp, H), H)
        out = sc.boundary(None, Tp, rr, w, 1e-5)
        res["sp_gemm_boundary_max_err"] = max((out.float() - want_full.float()).abs().max().item(),
                                              (rr.float() - want_res.float()).abs().max().item())
    torch.cuda.synchronize()
    keys = ("fused_allreduce_rmsnorm_max_err", "nvls_gemm_allreduce_rmsnorm_max_err", "sp_gemm_boundary_max_err")
    errs = torch.tensor([res.get(k, 0.0) for k in keys], device=dev)
    dist.all_reduce(errs, op=dist.ReduceOp.MAX)
    out = {k: round(errs[i].item(), 5) for i, k in enumerate(keys) if k in res}
    out["reference"] = ("NCCL all-reduce + fused_add_rms_norm kernel, [64, hidden] bf16; SP boundary: cuBLAS + "
                        "NCCL all-reduce, norm of this rank's rows, NCCL all-gather, [2048, hidden]; max over ranks")
    return out


class ClosedLoop:
    """Keeps ``C`` requests in flight through the public engine API: every finished request
    is replaced by a new prompt at once.  Records arrival / token timestamps per request."""

    def __init__(self, eng, vocab: int, C: int, P: int, O: int, seed: int = 1234):
        import torch

        from vllm_neuron_b200 import SamplingParams

        self.eng, self.C, self.P, self.O = eng, C, P, O
        self.SamplingParams = SamplingParams
        self.g = torch.Generator().manual_seed(seed)
        self.vocab = vocab
        self.n_added = 0
        self.arrival: dict[str, float] = {}
        self.first: dict[str, float] = {}
        self.seen: dict[str, int] = {}
        self.tok_times: dict[str, list[float]] = {}
        self.completions = 0

    def add(self, max_tokens: int) -> None:
        import torch

        rid = f"bench-{self.n_added}"
        self.n_added += 1
        prompt = torch.randint(0, self.vocab - 1000, (self.P,), generator=self.g).tolist()
        self.eng.add_request(rid, prompt, self.SamplingParams(temperature=0.0, max_tokens=max_tokens, ignore_eos=True))
        self.arrival[rid] = time.perf_counter()
        self.seen[rid] = 0

    def fill(self) -> None:
        """C requests with staggered output lengths (O/C, 2 O/C, ..., O): completions are evenly
        spread from the first decode step on, as in the steady state."""
        for i in range(self.C):
            self.add(max(1, (i + 1) * self.O // self.C))

    def step(self, record: bool) -> tuple[int, int]:
        """One engine step; returns (new output tokens, completions).  Replaces finished requests."""
        outs = self.eng.step()
        now = time.perf_counter()
        new_tok = done = 0
        for o in outs:
            rid = o.request_id
            n = len(o.outputs[0].token_ids)
            k = n - self.seen.get(rid, 0)
            if k > 0:
                new_tok += k
                self.seen[rid] = n
                if rid not in self.first:
                    self.first[rid] = now
                if record:
                    self.tok_times.setdefault(rid, []).extend([now] * k)
            if o.finished:
                done += 1
        self.completions += done
        for _ in range(done):
            self.add(self.O)
        return new_tok, done


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20, help="timed serving periods")
    ap.add_argument("--warmup", type=int, default=5, help="untimed serving periods")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--model", default="gpt-oss-120b", choices=["gpt-oss-120b", "gpt-oss-20b"])
    ap.add_argument("--concurrency", type=int, default=64)
    ap.add_argument("--prompt-len", type=int, default=2048)
    ap.add_argument("--output-len", type=int, default=512)
    ap.add_argument("--all2all", default="allgather_reducescatter",
                    help="EP token exchange at N > 1 (EngineConfig.all2all_backend)")
    ap.add_argument("--mixed-prefill-tokens", type=int, default=0,
                    help="prompt tokens per decode step (mixed steps); 0: separate prefill steps")
    ap.add_argument("--profile-dir", default=None,
                    help="also write a per-kernel table of one profiled serving period (rank 0)")
    ap.add_argument("--baseline-of-record", action="store_true",
                    help="the baseline of record: library GEMMs (cuBLAS) and NCCL collectives instead of the "
                         "tcgen05 GEMMs and fused NVLink / NVSwitch kernels (attention and MoE stay on this "
                         "framework's kernels: the reference's PyTorch MoE needs the experts dequantized to "
                         "bf16, ~234 GB for GPT-OSS-120B, which no single B200 holds)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    if args.baseline_of_record:
        os.environ["VLLM_B200_LIBRARY_GEMM"] = "1"
        os.environ["VLLM_B200_FUSED_COLLECTIVES"] = "0"
        os.environ["VLLM_B200_GEMM_ALLREDUCE"] = "0"
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")

    import torch
    import torch.distributed as dist

    from vllm_neuron_b200 import LLM

    N = args.gpus
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    hf = GPT_OSS_120B if args.model == "gpt-oss-120b" else GPT_OSS_20B
    C, P, O = args.concurrency, args.prompt_len, args.output_len
    max_len = P + O + 64
    t0 = time.time()
    llm = LLM(hf_config=hf, load_format="dummy", dtype="bfloat16", tensor_parallel_size=N,
              max_model_len=max_len, max_num_seqs=C, max_num_batched_tokens=4096, block_size=32,
              max_num_prefills_per_step=2, spmd=N > 1, seed=0, async_scheduling=True,
              mixed_prefill_tokens=args.mixed_prefill_tokens, all2all_backend=args.all2all,
              additional_config={"neuron_config": {"ep_degree": N, "quantization": "mxfp4",
                                                   "num_seqs_buckets": [C]}})
    eng = llm.engine
    runner = eng.worker.runner
    torch.cuda.synchronize()
    t_load = time.time() - t0

    def barrier():
        if dist.is_initialized():
            dist.barrier()
        torch.cuda.synchronize()

    coll_check = _collective_check(eng, hf["hidden_size"]) if N > 1 else None
    loop = ClosedLoop(eng, hf["vocab_size"], C, P, O)
    # ---- fill: C prompts prefilled back to back (the burst at the start of a serving run) ----
    loop.fill()
    t_pf = time.time()
    while any(r.num_computed_tokens < r.num_prompt_tokens for r in eng.scheduler.requests.values()):
        loop.step(False)
    torch.cuda.synchronize()
    t_fill = time.time() - t_pf
    if rank == 0:
        print(f"# load {t_load:.1f}s, fill prefill of {C}x{P} tokens {t_fill:.2f}s ({C * P / t_fill:.0f} tok/s)",
              file=sys.stderr)

    def run_periods(n: int, record: bool) -> tuple[int, list[int], list[int]]:
        """Steps until ``n`` more requests completed: (output tokens, h2d bytes, d2h bytes per step)."""
        tok, h2d, d2h = 0, [], []
        target = loop.completions + n
        while loop.completions < target:
            t, _ = loop.step(record)
            tok += t
            h2d.append(runner.h2d_bytes_last)
            d2h.append(runner.d2h_bytes_last)
        return tok, h2d, d2h

    # ---- warm-up periods (decode graph capture happens in the first decode step) ----
    run_periods(args.warmup, False)
    clocks = ClockSampler(local)
    barrier()
    clocks.start()
    # ---- timed window: K serving periods through the public engine API ----
    runner.step_spans = []
    window_start = time.perf_counter()
    arrivals_before = loop.n_added
    tokens, h2d, d2h = run_periods(args.steps, True)
    wall_s = time.perf_counter() - window_start
    torch.cuda.synchronize()
    spans = runner.step_spans
    runner.step_spans = None
    dev_ms = sum(a.elapsed_time(b) for a, b in spans)
    n_engine_steps = len(h2d)
    # TTFT of the requests that arrived in the window and got their first token in it
    window_ids = [f"bench-{i}" for i in range(arrivals_before, loop.n_added)]
    ttfts = sorted(loop.first[r] - loop.arrival[r] for r in window_ids if r in loop.first)
    # TPOT: per request, mean interval between its tokens after the first one seen in the window
    tpots = []
    for rid, ts in loop.tok_times.items():
        if len(ts) >= 3:
            tpots.append((ts[-1] - ts[0]) / (len(ts) - 1))
    tpots.sort()
    # ---- secondary: decode-only graph replays (device-timed, no prefill) ----
    key = next((k for k in runner.graphs if k[0] == C), None)
    dec_ms = float("nan")
    n_dec = 8 * args.steps
    if key is not None:
        graph = runner.graphs[key].graph
        for _ in range(3):
            graph.replay()
        barrier()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record()
        for _ in range(n_dec):
            graph.replay()
        e2.record()
        barrier()
        dec_ms = s2.elapsed_time(e2)
        del graph
    clk = clocks.stop()
    tms = torch.tensor([dev_ms, wall_s * 1000.0, dec_ms if key is not None else 0.0], dtype=torch.float64)
    if dist.is_initialized():
        t = tms.cuda()
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        tms = t.cpu()
    dev_ms, wall_ms, dec_ms = tms.tolist()
    # ---- kernel launches of this library per serving period (one profiled period after timing;
    # every rank runs it so the collectives stay matched) ----
    ours, total, table = _count_our_kernels(lambda: run_periods(1, False))
    launches = ours * args.steps
    if rank == 0 and args.profile_dir:
        os.makedirs(args.profile_dir, exist_ok=True)
        with open(os.path.join(args.profile_dir, f"serving_period_kernels_n{N}.txt"), "w") as f:
            f.write(f"# one serving period: {ours} launches of this library's kernels, {total} kernels in total\n")
            f.write(table)
    value = tokens / (dev_ms / 1000.0)
    base = BASELINE_OF_RECORD.get((args.model, N)) if not args.baseline_of_record else None
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": N, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dev_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": round(value / base, 3) if base else None,
            "dtype": "bf16 (experts MXFP4 weights, MXFP8 activations)",
            "data": "synthetic random prompt tokens; random-init weights (GPT-OSS-120B architecture)",
            "config": {"model": args.model, "global_batch": C, "seq_len": P, "output_len": O,
                       "parallelism": f"tp{N}-ep{N}" if N > 1 else "single",
                       "ep_exchange": args.all2all if N > 1 else None,
                       "collective_check": coll_check,
                       "phase": f"steady-state closed loop at concurrency {C}: each step is one serving period "
                                f"(a finished request replaced by a new {P}-token prompt, its prefill, and the "
                                f"decode steps until the next completion)",
                       "prefill_policy": (f"prompt chunks of <= {args.mixed_prefill_tokens} tokens inside the decode "
                                          f"steps (mixed steps)" if args.mixed_prefill_tokens
                                          else "separate prefill steps"),
                       "l2": "weights (~60 GB) and KV exceed L2 every engine step; no flush",
                       "output_tokens": tokens, "engine_steps": n_engine_steps,
                       "ttft_p50_ms": round(1000 * ttfts[len(ttfts) // 2], 2) if ttfts else None,
                       "tpot_p50_ms": round(1000 * tpots[len(tpots) // 2], 3) if tpots else None,
                       "requests_in_window": len(ttfts),
                       "decode_only_tok_s": round(C * n_dec / (dec_ms / 1000.0), 1) if key is not None else None,
                       "fill_prefill_tok_s": round(C * P / t_fill, 1)},
            "e2e": {"value": round(tokens / (wall_ms / 1000.0), 2), "unit": "tokens/s",
                    "api": "LLMEngine.add_request + LLMEngine.step (closed loop, wall clock)",
                    "h2d_bytes_per_step": int(statistics.mean(h2d)), "d2h_bytes_per_step": int(statistics.mean(d2h))},
            "gpu_launches": launches,
            "clocks": clk,
        }
        if args.baseline_of_record:
            line["impl"] = "baseline-of-record (cuBLAS GEMMs + NCCL collectives)"
        print(json.dumps(line))
        sys.stdout.flush()
    # Graphs that captured NCCL calls are freed before the process group is destroyed
    # (worker shutdown releases them, then destroys the groups); then a normal exit.
    runner.release_graphs()
    torch.cuda.synchronize()
    llm.shutdown()
    if dist.is_initialized():
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
