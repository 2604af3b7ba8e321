"""Headline benchmark: GPT-OSS-120B (MXFP4 experts) output tokens/s at concurrency 64.

``python bench.py --gpus N --steps K --warmup W`` (N > 1 under torch.distributed.run).

Workload (BASELINE.json config 3 shape): 64 concurrent requests of 2048 synthetic
random prompt tokens, random-init weights of the GPT-OSS-120B architecture (36 layers,
hidden 2880, 64 q / 8 kv heads of 64, 128 experts top-4, MXFP4 experts, bf16 rest).
All 64 prompts are prefilled through the engine, then decode runs at batch 64:
* ``value``  device-timed decode throughput: K replays of the captured decode step
  (forward + LM head + sampling for 64 sequences) between CUDA events, after W warm-up
  steps; tokens/s = 64 * K / t, t = max over ranks.  Weights (~60 GB) exceed L2, so no
  flush is needed between steps.
* ``e2e``    the same metric through the public engine API (``LLMEngine.step``, asynchronous
  scheduling): every step schedules, stages its inputs in pinned host memory, copies them
  H2D, replays the graph and reads the sampled ids back D2H (the host work of step k+1
  overlaps step k on the GPU).
Parallelism for N GPUs: attention TP=N (heads), experts EP=N, one all-reduce after
attention and one after the MoE per layer (NCCL); total concurrency stays 64 (strong
scaling).  ``--impl reference`` runs the reference plugin when it can run here.
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
    sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))
    reason = None
    try:
        import vllm_neuron.functional  # noqa: F401
    except Exception as e:  # noqa: BLE001
        reason = (f"reference installs from /root/reference but cannot run on B200: "
                  f"importing vllm_neuron.functional fails ({type(e).__name__}: {e}); it targets AWS Trainium "
                  f"(NKI kernels, neuronx-cc) and sets CUDA_VISIBLE_DEVICES='' at import")
    rank = int(os.environ.get("RANK", "0"))
    if rank == 0:
        print(json.dumps({"impl": "reference", "unavailable": reason or "reference has no CUDA execution path"}))


def _profile_replays(graph, n: int) -> tuple[int, int, str]:
    """Replay the decode graph n times under torch.profiler: (launches of this library's
    kernels per replay, all kernels per replay, per-kernel table)."""
    import torch

    acts = [torch.profiler.ProfilerActivity.CUDA]
    with torch.profiler.profile(activities=acts) as prof:
        for _ in range(n):
            graph.replay()
        torch.cuda.synchronize()
    ours = total = 0
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA:
            total += 1
            if "b200::" in ev.name:
                ours += 1
    table = prof.key_averages().table(sort_by="self_cuda_time_total", row_limit=40)
    return ours // n, total // n, table


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--model", default="gpt-oss-120b", choices=["gpt-oss-120b", "gpt-oss-20b"])
    ap.add_argument("--concurrency", type=int, default=64)
    ap.add_argument("--prompt-len", type=int, default=2048)
    ap.add_argument("--output-len", type=int, default=512)
    ap.add_argument("--profile-dir", default=None,
                    help="also write a per-kernel table of profiled decode-step replays (rank 0)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")

    import torch
    import torch.distributed as dist

    from vllm_neuron_b200 import LLM, SamplingParams

    N = args.gpus
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    hf = GPT_OSS_120B if args.model == "gpt-oss-120b" else GPT_OSS_20B
    C, P = args.concurrency, args.prompt_len
    max_len = P + args.output_len + 64
    t0 = time.time()
    llm = LLM(hf_config=hf, load_format="dummy", dtype="bfloat16", tensor_parallel_size=N,
              max_model_len=max_len, max_num_seqs=C, max_num_batched_tokens=4096, block_size=32,
              max_num_prefills_per_step=2, spmd=N > 1, seed=0, async_scheduling=True,
              additional_config={"neuron_config": {"ep_degree": N, "quantization": "mxfp4",
                                                   "num_seqs_buckets": [C]}})
    eng = llm.engine
    torch.cuda.synchronize()
    t_load = time.time() - t0
    g = torch.Generator().manual_seed(1234)
    prompts = [torch.randint(0, hf["vocab_size"] - 1000, (P,), generator=g).tolist() for _ in range(C)]
    sp = SamplingParams(temperature=0.0, max_tokens=args.output_len, ignore_eos=True)
    # ---- prefill all requests (TTFT per request from engine metrics) ----
    for i, p in enumerate(prompts):
        eng.add_request(f"bench-{i}", p, sp)
    t_pf = time.time()
    while any(r.num_computed_tokens < r.num_prompt_tokens for r in eng.scheduler.requests.values()):
        eng.step()
    torch.cuda.synchronize()
    t_prefill = time.time() - t_pf
    ttfts = sorted((r.metrics.first_token_time - r.metrics.arrival_time) for r in eng.scheduler.requests.values())
    ttft_p50 = ttfts[len(ttfts) // 2]
    runner = eng.worker.runner
    if rank == 0:
        print(f"# load {t_load:.1f}s prefill {t_prefill:.2f}s ({C * P / t_prefill:.0f} tok/s) ttft_p50 "
              f"{ttft_p50 * 1000:.1f} ms", file=sys.stderr)

    def barrier():
        if dist.is_initialized():
            dist.barrier()
        torch.cuda.synchronize()

    # ---- e2e through the public API: LLMEngine.step() (schedule, pinned H2D, replay, D2H) ----
    for _ in range(args.warmup):
        eng.step()
    clocks = ClockSampler(local)
    barrier()
    clocks.start()
    h2d, d2h = [], []
    s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0 = time.perf_counter()
    s_ev.record()
    for _ in range(args.steps):
        outs = eng.step()
        h2d.append(runner.h2d_bytes_last)
        d2h.append(runner.d2h_bytes_last)
    e_ev.record()
    barrier()
    e2e_wall = time.perf_counter() - w0
    e2e_ms = s_ev.elapsed_time(e_ev)
    # ---- device-timed decode step: replay the captured decode graph K times ----
    key = next(k for k in runner.graphs if k[0] == C) if runner.graphs else None
    if key is None:
        raise SystemExit("decode graph for the benchmark batch was not captured")
    graph = runner.graphs[key].graph
    for _ in range(args.warmup):
        graph.replay()
    barrier()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record()
    for _ in range(args.steps):
        graph.replay()
    e2.record()
    barrier()
    dev_ms = s2.elapsed_time(e2)
    clk = clocks.stop()
    tms = torch.tensor([dev_ms, e2e_ms, max(e2e_wall * 1000, e2e_ms)], dtype=torch.float64)
    if dist.is_initialized():
        t = tms.cuda()
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        tms = t.cpu()
    dev_ms, e2e_ms, e2e_wall_ms = tms.tolist()
    ms_step = dev_ms / args.steps
    value = C * args.steps / (dev_ms / 1000.0)
    e2e_val = C * args.steps / (e2e_wall_ms / 1000.0)
    tpot_ms = e2e_wall_ms / args.steps
    # kernel launches per decode step, counted from one profiled replay after the timed region
    # (every rank replays so the graphs' collectives stay matched)
    ours, total, table = _profile_replays(graph, 1 if not args.profile_dir else 5)
    launches = ours * args.steps
    if rank == 0 and args.profile_dir:
        os.makedirs(args.profile_dir, exist_ok=True)
        with open(os.path.join(args.profile_dir, f"decode_step_kernels_n{N}.txt"), "w") as f:
            f.write(f"# {ours} launches of this library's kernels, {total} kernels in total, per decode step\n")
            f.write(table)
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": N, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16 (experts MXFP4 weights, MXFP8 activations)",
            "data": "synthetic random prompt tokens; random-init weights (GPT-OSS-120B architecture)",
            "config": {"model": args.model, "global_batch": C, "seq_len": P, "output_len": args.output_len,
                       "parallelism": f"tp{N}-ep{N}" if N > 1 else "single", "phase": "decode at concurrency "
                       f"{C} after prefilling {C}x{P} tokens", "l2": "weights per step (~60 GB) exceed L2; no flush",
                       "ttft_p50_ms": round(ttft_p50 * 1000, 2), "tpot_p50_ms": round(tpot_ms, 3),
                       "prefill_tok_s": round(C * P / t_prefill, 1)},
            "e2e": {"value": round(e2e_val, 2), "unit": "tokens/s", "api": "LLMEngine.step",
                    "h2d_bytes_per_step": int(statistics.mean(h2d)), "d2h_bytes_per_step": int(statistics.mean(d2h))},
            "gpu_launches": launches,
            "clocks": clk,
        }
        print(json.dumps(line))
    # Graphs that captured NCCL calls must be freed before the process group is destroyed,
    # including the local reference taken above; then leave without interpreter teardown.
    del graph
    runner.release_graphs()
    torch.cuda.synchronize()
    sys.stdout.flush()
    llm.shutdown()
    sys.stdout.flush()
    os._exit(0)


if __name__ == "__main__":
    main()
