"""The no-allocation decode-attention entry point, called through its exported C symbol.

Callers that cannot allocate device memory (a C runtime without an allocator handle, or a
process whose device memory another allocator has already reserved) use
``b200_paged_attention_decode_noalloc``: it takes only inputs and outputs and keeps its
split-KV partials in a fixed array inside the library.  This test checks its output against
the regular entry point (``torch.ops.b200.paged_attention_decode`` with a caller-provided
workspace) on two calls in a row that both use the shared array, and that oversized or
malformed requests are refused.  The file is
named so that pytest collects it last."""

import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"
SCRATCH_TOO_SMALL = 1005  # kScratchTooSmall (csrc/common.cuh)
BAD_SHAPE = 1003  # kBadShape


def _lib():
    from vllm_neuron_b200.ops._ext import load, so_path

    assert load(), "CUDA extension must be built in-tree"
    lib = ctypes.CDLL(so_path())
    fn = lib.b200_paged_attention_decode_noalloc
    P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    fn.argtypes = [P, P, P, P, P, P, P, I, I, I, I, I, I, I, I, F, F, F, I, I, I, P]
    fn.restype = ctypes.c_int
    return fn


def _case(seed, seq_lens=(1, 40, 700, 2049, 5000), nq=16, nkv=2):
    g = torch.Generator(device="cpu").manual_seed(seed)
    seq_lens = list(seq_lens)
    B, d, bs = len(seq_lens), 64, 32
    max_blocks = max(math.ceil(s / bs) for s in seq_lens)
    nb = sum(math.ceil(s / bs) for s in seq_lens) + 1
    perm = torch.randperm(nb - 1, generator=g) + 1
    bt = torch.zeros(B, max_blocks, dtype=torch.int32)
    off = 0
    for i, s in enumerate(seq_lens):
        n = math.ceil(s / bs)
        bt[i, :n] = perm[off:off + n]
        off += n
    kc = torch.randn(nb, nkv, bs, d, generator=g).bfloat16().to(DEV)
    vc = torch.randn(nb, nkv, bs, d, generator=g).bfloat16().to(DEV)
    q = torch.randn(B, nq, d, generator=g).bfloat16().to(DEV)
    sinks = torch.randn(nq, generator=g).to(DEV)
    return q, kc, vc, bt.to(DEV), torch.tensor(seq_lens, dtype=torch.int32, device=DEV), sinks


def _call(fn, out, q, kc, vc, bt, sl, sinks, splits, window, scale):
    B, nq, d = q.shape
    stream = torch.cuda.current_stream().cuda_stream
    return fn(out.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), sl.data_ptr(),
              sinks.data_ptr(), B, nq, kc.shape[1], d, q.stride(0), kc.shape[2], bt.stride(0), window, scale,
              1.0, 1.0, splits, 2, 2, stream)  # dtype / cache dtype 2 = bf16


def test_noalloc_matches_workspace_entry_point_twice():
    """Two calls in a row whose split counts (5, then 3) both merge through the shared
    scratch array, with different shapes, so the second call runs on whatever the first
    one left there."""
    fn = _lib()
    scale = 64 ** -0.5
    cases = [(0, 5, 0, (1, 40, 700, 2049, 5000), 16, 2), (1, 3, 128, (3000, 17, 260), 8, 1)]
    for call, (seed, splits, window, lens, nq, nkv) in enumerate(cases):
        q, kc, vc, bt, sl, sinks = _case(seed, lens, nq, nkv)
        B, nq, d = q.shape
        ws = torch.empty(B * nq * splits * (d + 1), device=DEV)
        want = torch.empty_like(q)
        torch.ops.b200.paged_attention_decode(want, q, kc, vc, bt, sl, sinks, window, scale, 1.0, 1.0, ws, splits)
        got = torch.full_like(q, float("nan"))
        rc = _call(fn, got, q, kc, vc, bt, sl, sinks, splits, window, scale)
        assert rc == 0, f"call {call}: return code {rc}"
        torch.cuda.synchronize()
        err = (got.float() - want.float()).abs().max().item()
        assert err <= 1e-2, f"call {call}: max abs difference {err}"


def test_noalloc_rejects_bad_shape():
    fn = _lib()
    q, kc, vc, bt, sl, sinks = _case(3)
    out = torch.empty_like(q)
    B, nq, d = q.shape
    stream = torch.cuda.current_stream().cuda_stream
    for nkv in (0, 3):  # no kv heads; query heads not a multiple of the kv heads
        rc = fn(out.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), sl.data_ptr(),
                sinks.data_ptr(), B, nq, nkv, d, q.stride(0), kc.shape[2], bt.stride(0), 0, 0.125, 1.0, 1.0, 5,
                2, 2, stream)
        assert rc == BAD_SHAPE


def test_noalloc_rejects_oversized_request():
    fn = _lib()
    q, kc, vc, bt, sl, sinks = _case(2)
    big_splits = 4096  # 5 * 16 * 4096 * 65 floats > the 4 MiB scratch
    out = torch.empty_like(q)
    rc = _call(fn, out, q, kc, vc, bt, sl, sinks, big_splits, 0, 0.125)
    assert rc == SCRATCH_TOO_SMALL
