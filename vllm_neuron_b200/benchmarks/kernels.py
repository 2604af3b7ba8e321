"""Kernel microbenchmarks on serving shapes (one GPU).

``python -m vllm_neuron_b200.benchmarks.kernels --op moe_mxfp4 --iters 20``

Each op is timed with CUDA events on the launching stream after warm-up, with a read of
a buffer larger than L2 between timed iterations (so every iteration reads its operands
from HBM and no dirty lines are left to write back inside the timed region), and reported as one JSON line: mean milliseconds, the algorithmic bytes and
FLOPs of one call, achieved GB/s and TFLOP/s, and the fraction of the measured copy
bandwidth / bf16 GEMM peak (``MEASURED_PEAKS.json`` at the repository root, if present).
The same command with ``--iters 1 --warmup 1`` is the small case for a profiler capture.

Shapes (defaults are the GPT-OSS-120B decode step at concurrency 64 and the Qwen3-Next
layer shapes at TP=4):
  moe_mxfp4    T=64 tokens x top-4 over 128 MXFP4 experts, H = I = 2880 (one MoE layer)
  moe_bf16     T=64, 16 bf16 experts, H = I = 2880
  attn_decode  B=64 sequences x 2048 context, 64 q / 8 kv heads, d=64, bf16 paged cache
  attn_prefill 1 x 2048-token prompt, 64 q / 8 kv heads, d=64
  gdn_prefill  8192-token prompt, 4 key / 8 value heads of 128 (Qwen3-Next TP=4)
  gdn_decode   64 sequences, 8 value heads of 128
  kv_transfer  one 2048-token GPT-OSS-120B request: device export + import (disaggregated serving)
  gemm         y[T, N] = x[T, K] W^T (+ fp32 out with --fp32-out): the tcgen05 dense GEMM of every
               linear layer; --library times torch.nn.functional.linear (cuBLAS) on the same shape.
               Default 64 x 5120 x 2880 (GPT-OSS QKV at TP=1); LM head: --T 64 --N 201088 --K 2880
"""

from __future__ import annotations

import argparse
import json
import os
import statistics

import torch


def _peaks() -> dict:
    here = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    try:
        with open(os.path.join(here, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "fallback": True}


def _graphed(fn):
    """Capture ``fn`` into a CUDA graph (as the engine's decode step runs), so the timed
    region holds device work only: eager launches of a multi-kernel op spend ~20 us of
    host time per call, more than a small kernel's device time.  Returns (replay, mode)."""
    try:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            fn()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        torch.cuda.synchronize()
        return g.replay, "graph"
    except Exception:  # an op with a host sync cannot be captured: time it eagerly
        torch.cuda.synchronize()
        return fn, "eager"


def _time(fn, iters: int, warmup: int, flush: torch.Tensor) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        # evict L2 by READING a buffer larger than it (126 MB): a write flush leaves ~126 MB
        # of dirty lines whose write-back then lands inside the timed kernel (~19 us at HBM
        # speed, most of a small kernel's time); after a read every resident line is clean
        flush.sum()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    # event timestamps on this part tick in ~2 us steps, so a median of short kernels snaps
    # to the grid; the mean over many iterations (random phase) is not quantised
    return statistics.fmean(times)


def _moe_mxfp4(args):
    from vllm_neuron_b200 import ops
    from vllm_neuron_b200.ops.mx_layout import scales_to_atoms, tile_values

    T, E, H, I, k = args.T or 64, args.E or 128, 2880, 2880, 4
    dev = "cuda"
    x = torch.randn(T, H, device=dev).bfloat16()
    w13 = tile_values(torch.randint(0, 256, (E, 2 * I, H // 2), device=dev, dtype=torch.uint8), H)
    s13 = scales_to_atoms(torch.full((E, 2 * I, H // 32), 120, device=dev, dtype=torch.uint8), H)
    w2 = tile_values(torch.randint(0, 256, (E, H, I // 2), device=dev, dtype=torch.uint8), I)
    s2 = scales_to_atoms(torch.full((E, H, I // 32), 120, device=dev, dtype=torch.uint8), I)
    b13 = torch.zeros(E, 2 * I, device=dev)
    b2 = torch.zeros(E, H, device=dev)
    v, ids = torch.topk(torch.randn(T, E, device=dev), k, -1)
    wts = torch.softmax(v, -1)
    ids = ids.to(torch.int32)
    touched = int(torch.unique(ids).numel())
    nbytes = touched * (2 * I * H // 2 + H * I // 2) * 1.0625 + T * H * 4  # fp4 values + ue8m0 scales + x/out
    flops = 2 * T * k * (2 * I * H + H * I)
    fn = lambda: ops.moe_mxfp4(x, ids, wts, w13, s13, b13, w2, s2, b2, 0, 1.702, 7.0, H, I)  # noqa: E731
    return fn, nbytes, flops, {"T": T, "E": E, "H": H, "I": I, "k": k, "experts_touched": touched}


def _moe_bf16(args):
    from vllm_neuron_b200 import ops

    T, E, H, I, k = args.T or 64, args.E or 16, 2880, 2880, 4
    dev = "cuda"
    x = torch.randn(T, H, device=dev).bfloat16()
    w13 = (torch.randn(E, 2 * I, H, device=dev) * 0.02).bfloat16()
    w2 = (torch.randn(E, H, I, device=dev) * 0.02).bfloat16()
    t13, t2 = ops.prepare_moe_bf16(w13, w2, True)
    del w13, w2
    v, ids = torch.topk(torch.randn(T, E, device=dev), k, -1)
    wts = torch.softmax(v, -1)
    ids = ids.to(torch.int32)
    touched = int(torch.unique(ids).numel())
    nbytes = touched * (2 * I * H + H * I) * 2 + T * H * 4
    flops = 2 * T * k * (2 * I * H + H * I)
    fn = lambda: ops.moe_dense(x, ids, wts, t13, None, t2, None, 0, 1.702, 7.0, True, "swiglu_clamp", H, I)  # noqa
    return fn, nbytes, flops, {"T": T, "E": E, "H": H, "I": I, "k": k, "experts_touched": touched}


def _paged(B, L, hq, hkv, d, bs=32):
    dev = "cuda"
    nb_per = (L + bs - 1) // bs
    nb = B * nb_per + 1
    kc = torch.randn(nb, hkv, bs, d, device=dev).bfloat16()
    vc = torch.randn(nb, hkv, bs, d, device=dev).bfloat16()
    bt = (torch.arange(B * nb_per, device=dev, dtype=torch.int32) + 1).view(B, nb_per)
    sl = torch.full((B,), L, dtype=torch.int32, device=dev)
    return kc, vc, bt, sl


def _attn_decode(args):
    from vllm_neuron_b200 import ops
    from vllm_neuron_b200.ops.metadata import AttentionMetadata

    B, L, d = args.T or 64, args.L or 2048, 64
    hq, hkv = args.hq or 64, args.hkv or 8
    kc, vc, bt, sl = _paged(B, L, hq, hkv, d)
    q = torch.randn(B, hq, d, device="cuda").bfloat16()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    from vllm_neuron_b200.engine.model_runner import decode_splits

    splits = args.splits or decode_splits(B, hkv, sms)
    ws = torch.empty(B * hq * splits * (d + 2), device="cuda")
    qsl = torch.arange(B + 1, dtype=torch.int32, device="cuda")
    meta = AttentionMetadata(B, B, True, qsl, sl, bt, None, None, 1, L, workspace=ws, num_splits=splits)
    nbytes = 2 * B * L * hkv * d * 2 + 2 * B * hq * d * 2
    flops = 4 * B * hq * L * d
    fn = lambda: ops.attention(q, kc, vc, meta, d ** -0.5)  # noqa: E731
    return fn, nbytes, flops, {"B": B, "L": L, "hq": hq, "hkv": hkv, "d": d, "splits": splits}


def _mla_decode(args):
    """MLA decode (absorbed): B sequences of L tokens, hq heads (default 16: 128 heads over
    TP 8), latent cache rows of 576 bf16 in 64-token blocks."""
    from vllm_neuron_b200 import ops

    B, L, hq, bs = args.T or 64, args.L or 2048, args.hq or 16, 64
    nb = -(-L // bs)
    cache = (torch.randn(B * nb, bs, 576, device="cuda") * 0.5).bfloat16()
    bt = torch.randperm(B * nb, device="cuda").to(torch.int32).reshape(B, nb)
    sl = torch.full((B,), L, dtype=torch.int32, device="cuda")
    q = torch.randn(B, hq, 576, device="cuda").bfloat16()
    splits = args.splits or None
    nbytes = B * L * 576 * 2 + B * hq * (576 + 512) * 2
    flops = 2 * B * hq * L * (576 + 512)
    fn = lambda: ops.mla_decode(q, cache, bt, sl, 192 ** -0.5, num_splits=splits, max_seq_len=L)  # noqa: E731
    return fn, nbytes, flops, {"B": B, "L": L, "hq": hq, "block": bs, "splits": splits or "auto"}


def _attn_prefill(args):
    from vllm_neuron_b200 import ops
    from vllm_neuron_b200.ops.metadata import AttentionMetadata

    L, hq, hkv, d = args.L or 2048, args.hq or 64, args.hkv or 8, 64
    kc, vc, bt, sl = _paged(1, L, hq, hkv, d)
    q = torch.randn(L, hq, d, device="cuda").bfloat16()
    qsl = torch.tensor([0, L], dtype=torch.int32, device="cuda")
    meta = AttentionMetadata(L, 1, False, qsl, sl, bt, None, None, L, L)
    nbytes = 2 * L * hkv * d * 2 + 2 * L * hq * d * 2
    flops = 2 * hq * L * L * d  # causal: half of 4*L*L*d per head
    fn = lambda: ops.attention(q, kc, vc, meta, d ** -0.5)  # noqa: E731
    return fn, nbytes, flops, {"L": L, "hq": hq, "hkv": hkv, "d": d}


def _gemm(args):
    import torch.nn.functional as F

    from vllm_neuron_b200 import ops

    T, N, K = args.T or 64, args.N or 5120, args.K or 2880
    x = torch.randn(T, K, device="cuda").bfloat16()
    w = (torch.randn(N, K, device="cuda") * 0.02).bfloat16()
    out_dtype = torch.float32 if args.fp32_out else None
    if args.library:
        fn = lambda: F.linear(x, w)  # noqa: E731
    else:
        fn = lambda: ops.linear(x, w, None, out_dtype)  # noqa: E731
    nbytes = N * K * 2 + T * K * 2 + T * N * (4 if args.fp32_out else 2)
    return fn, nbytes, 2 * T * N * K, {"T": T, "N": N, "K": K, "impl": "cublas" if args.library else "tcgen05"}


def _gdn(args, decode: bool):
    from vllm_neuron_b200 import ops
    from vllm_neuron_b200.ops.metadata import AttentionMetadata

    nk, nv, d = 4, 8, 128
    if decode:
        B = args.T or 64
        lens = [1] * B
    else:
        B, lens = 1, [args.L or 8192]
    T = sum(lens)
    dev = "cuda"
    qsl = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32, device=dev)
    meta = AttentionMetadata(T, B, decode, qsl, None, None, None, None, max(lens), max(lens))
    meta.extras = {"state_slots": torch.arange(B, dtype=torch.int32, device=dev),
                   "state_init": torch.ones(B, dtype=torch.int32, device=dev)}
    mixed = torch.randn(T, 2 * nk * d + nv * d, device=dev).bfloat16()
    proj = torch.randn(T, nv * d + 2 * nv, device=dev).bfloat16()
    z, b, a = proj[:, :nv * d], proj[:, nv * d:nv * d + nv], proj[:, nv * d + nv:]
    A_log = torch.zeros(nv, device=dev)
    dt = torch.zeros(nv, device=dev)
    nw = torch.ones(d, device=dev)
    state = torch.zeros(B, nv, d, d, device=dev)
    nbytes = 2 * state.numel() * 4 + mixed.numel() * 2 + proj.numel() * 2 + T * nv * d * 2
    chunks = -(-T // 64)
    flops = (2 * T * nv * d * d * 4 + chunks * nv * 2 * 64 * 64 * d * 4) if not decode else 6 * T * nv * d * d
    fn = lambda: ops.gated_delta_net(mixed, z, b, a, A_log, dt, nw, 1e-6, state, meta, nk, nv, d, d)  # noqa
    return fn, nbytes, flops, {"T": T, "B": B, "nk": nk, "nv": nv, "d": d}


def _kv_transfer(args):
    """Device KV transfer of one request (disaggregated serving): export from a paged cache
    into a device pool + import into another cache (same GPU here; the decode engine reads the
    pool over NVLink when it sits on another GPU).  GPT-OSS-120B shape at TP=1: 36 layers,
    8 kv heads of 64, 2048 tokens, bf16."""
    from vllm_neuron_b200.ops import _ext

    _ext.load()
    ops = torch.ops.b200
    L, T, nh, d, bs = 36, args.L or 2048, 8, 64, 32
    nb = T // bs
    dev = "cuda"
    src = [(torch.randn(nb + 1, nh, bs, d, device=dev).bfloat16(), torch.randn(nb + 1, nh, bs, d, device=dev).bfloat16())
           for _ in range(L)]
    dst = [(torch.zeros_like(k), torch.zeros_like(v)) for k, v in src]
    kp = torch.tensor([k.data_ptr() for k, _ in src], dtype=torch.int64, device=dev)
    vp = torch.tensor([v.data_ptr() for _, v in src], dtype=torch.int64, device=dev)
    kq = torch.tensor([k.data_ptr() for k, _ in dst], dtype=torch.int64, device=dev)
    vq = torch.tensor([v.data_ptr() for _, v in dst], dtype=torch.int64, device=dev)
    blocks = torch.randperm(nb, device=dev).to(torch.int32) + 1
    region = 2 * L * T * nh * d * 2
    pool = ops.comm_alloc(region // 2 + 256)
    base = pool + 64 * 1024
    row = d * 2

    keep = (src, dst)  # the pointer tables hold raw addresses: the caches must outlive fn

    def fn(_keep=keep):
        ops.kv_export(base, kp, vp, blocks, T, nh, row, bs)
        ops.kv_import([base], [0], [nh], kq, vq, blocks, T, T, 0, nh, row, bs, None)

    fn()
    torch.cuda.synchronize()
    k0 = src[5][0][blocks.long()].permute(0, 2, 1, 3)
    assert torch.equal(k0, dst[5][0][blocks.long()].permute(0, 2, 1, 3)), "kv transfer mismatch"
    return fn, 4 * region, 0, {"layers": L, "tokens": T, "kv_heads": nh, "d": d, "request_bytes": region}


OPS = {
    "kv_transfer": _kv_transfer,
    "moe_mxfp4": _moe_mxfp4,
    "moe_bf16": _moe_bf16,
    "attn_decode": _attn_decode,
    "mla_decode": _mla_decode,
    "attn_prefill": _attn_prefill,
    "gemm": _gemm,
    "gdn_prefill": lambda a: _gdn(a, False),
    "gdn_decode": lambda a: _gdn(a, True),
}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", choices=sorted(OPS) + ["all"], default="all")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--T", type=int, default=0, help="tokens / sequences (op-specific)")
    ap.add_argument("--E", type=int, default=0, help="experts")
    ap.add_argument("--L", type=int, default=0, help="context / prompt length")
    ap.add_argument("--splits", type=int, default=0, help="split-KV factor for attn_decode (0 = heuristic)")
    ap.add_argument("--hq", type=int, default=0, help="query heads (attention ops; default 64)")
    ap.add_argument("--hkv", type=int, default=0, help="kv heads (attention ops; default 8)")
    ap.add_argument("--N", type=int, default=0, help="gemm output features")
    ap.add_argument("--K", type=int, default=0, help="gemm input features")
    ap.add_argument("--fp32-out", action="store_true", help="gemm with fp32 output (router logits)")
    ap.add_argument("--library", action="store_true", help="gemm through cuBLAS instead of the tcgen05 kernel")
    ap.add_argument("--eager", action="store_true", help="time eager launches instead of a CUDA-graph replay")
    args = ap.parse_args()
    peaks = _peaks()
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")  # 256 MB > L2
    names = sorted(OPS) if args.op == "all" else [args.op]
    with torch.inference_mode():
        for name in names:
            fn, nbytes, flops, shape = OPS[name](args)
            run, mode = (fn, "eager") if args.eager else _graphed(fn)
            ms = _time(run, args.iters, args.warmup, flush)
            gbs = nbytes / ms / 1e6
            tfl = flops / ms / 1e9
            print(json.dumps({"op": name, "ms": round(ms, 4), "bytes": int(nbytes), "flops": int(flops),
                              "GB/s": round(gbs, 1), "TFLOP/s": round(tfl, 2),
                              "frac_hbm": round(gbs / peaks["hbm_gbs"], 3),
                              "frac_bf16_peak": round(tfl / peaks["bf16_tflops"], 3),
                              "peaks": "fallback" if peaks.get("fallback") else "measured", "timing": mode,
                              "shape": shape}),
                  flush=True)
            del fn, run
            torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
