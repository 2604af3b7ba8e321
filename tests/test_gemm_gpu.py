"""The tcgen05 dense GEMM (``csrc/gemm.cu``) against an fp32 PyTorch reference of the same op,
and its fused all-reduce epilogue.

The fused all-reduce is checked on one GPU without any cross-GPU wait: two "ranks" are two
producer calls (different activations and weight shards) that add into one local region
(global atomics instead of multimem), then the finish kernel expects both ranks' tiles.
Three rounds in a row cover the parity flip of the double-buffered counters / accumulators
and the zeroing done by the finish kernel."""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _ref(x, w, b):
    y = x.float() @ w.float().t()
    return y + b.float() if b is not None else y


def _close(got, want, what):
    err = (got.float() - want).abs()
    tol = 8e-3 * want.abs() + 2e-3 * want.abs().max() + 1e-3
    bad = (err > tol).sum().item()
    assert bad == 0, f"{what}: {bad} elements off, max err {err.max().item():.4g} (max |ref| {want.abs().max().item():.3g})"


@pytest.mark.parametrize("T,N,K", [(1, 128, 64), (5, 640, 2880), (16, 2880, 512), (33, 5120, 2880),
                                   (64, 2880, 4096), (64, 25136, 2880), (100, 1000, 360), (300, 2048, 1024),
                                   (2048, 2880, 2880), (130, 136, 4104),
                                   # token tiles of 160 / 224 / 192 from the wave-balancing planner
                                   (900, 2880, 1024), (1200, 2880, 512), (1500, 2048, 640)])
def test_gemm_matches_fp32(T, N, K):
    from vllm_neuron_b200 import ops

    g = torch.Generator(device="cpu").manual_seed(T * 7 + N + K)
    x = (torch.randn(T, K, generator=g) * 0.5).bfloat16().to(DEV)
    w = (torch.randn(N, K, generator=g) * 0.05).bfloat16().to(DEV)
    b = (torch.randn(N, generator=g) * 0.1).bfloat16().to(DEV)
    for bias in (b, None):
        y = ops.linear(x, w, bias)
        torch.cuda.synchronize()
        assert y.shape == (T, N) and y.dtype == torch.bfloat16
        _close(y, _ref(x, w, bias), f"T={T} N={N} K={K} bias={bias is not None}")
    assert ops.check_device_status(x.device) == 0


def test_gemm_lm_head_shape_and_strided_input():
    """The GPT-OSS LM head (vocab 201088 x 2880) at decode batch 64, and an input that is a
    column slice of a wider tensor (row stride > K)."""
    from vllm_neuron_b200 import ops

    g = torch.Generator(device="cpu").manual_seed(5)
    wide = (torch.randn(64, 4096, generator=g) * 0.5).bfloat16().to(DEV)
    x = wide[:, 128:128 + 2880]
    w = (torch.randn(201088, 2880, generator=g) * 0.02).bfloat16().to(DEV)
    y = ops.linear(x, w)
    torch.cuda.synchronize()
    _close(y, _ref(x, w, None), "lm head")


def test_gemm_split_k_repeated_calls():
    """Split K (few output tiles, long K): the per-tile counters return to zero, so repeated
    calls with changing inputs stay correct."""
    from vllm_neuron_b200 import ops

    g = torch.Generator(device="cpu").manual_seed(9)
    w = (torch.randn(256, 8192, generator=g) * 0.02).bfloat16().to(DEV)
    ws, cnt = ops._gemm_workspace(torch.device(DEV))
    for i in range(4):
        x = (torch.randn(8 + i, 8192, generator=g)).bfloat16().to(DEV)
        _close(ops.linear(x, w), _ref(x, w, None), f"call {i}")
    torch.cuda.synchronize()
    assert int(cnt.abs().sum().item()) == 0
    assert ws.abs().max().item() == 0.0  # the scratch sums were cleared by the last splits


def _finish_ref(parts, bias, residual, nw, eps):
    s = sum(parts)
    if bias is not None:
        s = s + bias.float()
    s_bf = s.bfloat16().float()
    new_res = (s_bf + residual.float()).bfloat16()
    r = new_res.float()
    out = r * torch.rsqrt(r.pow(2).mean(-1, keepdim=True) + eps) * nw
    return out, new_res


@pytest.mark.parametrize("T", [1, 64, 200])
def test_gemm_allreduce_two_emulated_ranks(T):
    ops = torch.ops.b200
    H, Kr, T_cap, H_cap, eps = 2880, 512, 256, 4096, 1e-5
    region = torch.zeros(int(ops.red_region_bytes(T_cap, H_cap)), dtype=torch.uint8, device=DEV)
    status = torch.zeros(4, dtype=torch.int32, device=DEV)
    g = torch.Generator(device="cpu").manual_seed(T)
    nw = (1 + 0.1 * torch.randn(H, generator=g)).float().to(DEV)
    bias = (0.1 * torch.randn(H, generator=g)).bfloat16().to(DEV)
    residual = torch.randn(T, H, generator=g).bfloat16().to(DEV)
    for rnd in range(3):
        xs = [torch.randn(T, Kr, generator=g).bfloat16().to(DEV) for _ in range(2)]
        ws = [(0.05 * torch.randn(H, Kr, generator=g)).bfloat16().to(DEV) for _ in range(2)]
        items = [ops.gemm_bf16_allreduce(x, w, region.data_ptr(), 0, T_cap, H_cap, 2, status)
                 for x, w in zip(xs, ws)]
        want_out, want_res = _finish_ref([_ref(x, w, None) for x, w in zip(xs, ws)], bias, residual, nw, eps)
        out = torch.empty(T, H, dtype=torch.bfloat16, device=DEV)
        ops.allreduce_finish(region.data_ptr(), T_cap, H_cap, sum(items), out, residual, bias, nw, eps, 64, status,
                             1_000_000_000)
        torch.cuda.synchronize()
        assert int(status[0].item()) == 0, f"round {rnd}: status {status.tolist()}"
        assert (residual.float() - want_res.float()).abs().max().item() <= 0.05 * want_res.float().abs().max().item()
        _close(out, want_out, f"round {rnd}")
        residual = want_res.clone()  # continue from the exact reference residual
    # every accumulator is zero again and both counters are reset
    hdr = region[:8].view(torch.int32)
    assert hdr.tolist() == [0, 0]
    assert region[256:].view(torch.float32).abs().max().item() == 0.0


def test_gemm_allreduce_plain_sum():
    """The finish kernel without a norm weight: out = sum + bias."""
    ops = torch.ops.b200
    T, H, Kr, T_cap, H_cap = 8, 1024, 256, 64, 1024
    region = torch.zeros(int(ops.red_region_bytes(T_cap, H_cap)), dtype=torch.uint8, device=DEV)
    g = torch.Generator(device="cpu").manual_seed(3)
    x = torch.randn(T, Kr, generator=g).bfloat16().to(DEV)
    w = (0.05 * torch.randn(H, Kr, generator=g)).bfloat16().to(DEV)
    b = (0.1 * torch.randn(H, generator=g)).bfloat16().to(DEV)
    n = ops.gemm_bf16_allreduce(x, w, region.data_ptr(), 0, T_cap, H_cap, 4, None)
    out = torch.empty(T, H, dtype=torch.bfloat16, device=DEV)
    ops.allreduce_finish(region.data_ptr(), T_cap, H_cap, n, out, None, b, None, 0.0, 8, None)
    torch.cuda.synchronize()
    _close(out, _ref(x, w, b), "plain sum")


@pytest.mark.parametrize("T,N", [(64, 128), (2048, 128), (7, 512)])
def test_gemm_fp32_output(T, N):
    """Router logits: fp32 straight from the accumulator (with and without split K)."""
    from vllm_neuron_b200 import ops

    g = torch.Generator(device="cpu").manual_seed(T + N)
    x = torch.randn(T, 2880, generator=g).bfloat16().to(DEV)
    w = (torch.randn(N, 2880, generator=g) * 0.02).bfloat16().to(DEV)
    b = (torch.randn(N, generator=g) * 0.1).bfloat16().to(DEV)
    y = ops.linear(x, w, b, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert y.dtype == torch.float32
    want = _ref(x, w, b)
    assert (y - want).abs().max().item() <= 1e-3 * want.abs().max().item() + 1e-4
