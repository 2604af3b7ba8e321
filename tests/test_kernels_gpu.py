"""Numerics of every sm_100a kernel against the fp32 PyTorch reference of the same op."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

from vllm_neuron_b200 import ops  # noqa: E402
from vllm_neuron_b200.ops import reference as ref  # noqa: E402
from vllm_neuron_b200.ops._ext import load, so_path  # noqa: E402
from vllm_neuron_b200.ops.metadata import AttentionMetadata  # noqa: E402

DEV = "cuda"


def _close(a, b, atol, rtol, what=""):
    a, b = a.float(), b.float()
    err = (a - b).abs()
    tol = atol + rtol * b.abs()
    bad = (err > tol).sum().item()
    assert bad == 0, f"{what}: {bad} mismatches, max err {err.max().item():.4g} (ref max {b.abs().max().item():.4g})"


def test_extension_loaded():
    assert load(), "CUDA extension must be built in-tree"
    assert so_path() and so_path().endswith(".so")


@pytest.mark.parametrize("H", [256, 2880, 5120])
def test_rms_norm(H):
    torch.manual_seed(0)
    x = torch.randn(37, H, device=DEV, dtype=torch.bfloat16)
    w = torch.rand(H, device=DEV) + 0.5
    _close(ops.rms_norm(x, w, 1e-5), ref.rms_norm(x.float(), w, 1e-5), 2e-2, 2e-2, "rms_norm")
    r = torch.randn_like(x)
    r0 = r.clone()
    out, r1 = ops.fused_add_rms_norm(x, r, w, 1e-5)
    want, wr = ref.fused_add_rms_norm(x.float(), r0.float(), w, 1e-5)
    _close(r1, wr, 2e-2, 1e-2, "residual")
    _close(out, want, 3e-2, 3e-2, "fused norm")


def test_embedding():
    w = torch.randn(1000, 2880, device=DEV, dtype=torch.bfloat16)
    ids = torch.tensor([0, 5, 999, 1000, 1500, 7], device=DEV)
    got = ops.embedding(ids, w, 500)
    loc = ids - 500
    exp = torch.where(((loc >= 0) & (loc < 1000))[:, None], w[loc.clamp(0, 999)], torch.zeros_like(w[:1]))
    assert torch.equal(got, exp)


@pytest.mark.parametrize("d,nq,nkv,rd,qknorm", [(64, 8, 1, 64, False), (128, 8, 2, 128, True), (256, 4, 2, 64, True)])
def test_rope_kv_write(d, nq, nkv, rd, qknorm):
    torch.manual_seed(1)
    T, bs, nb = 23, 16, 10
    qkv = torch.randn(T, (nq + 2 * nkv) * d + 8, device=DEV, dtype=torch.bfloat16)[:, : (nq + 2 * nkv) * d]
    pos = torch.randint(0, 4000, (T,), device=DEV)
    inv, af = ref.yarn_inv_freq(rd, 150000.0, 32.0, 4096)
    cs = ops.build_cos_sin_cache(inv, 4096, af, device=DEV)
    slots = torch.randperm(nb * bs, device=DEV)[:T]
    slots[3] = -1
    qn = torch.rand(d, device=DEV) + 0.5 if qknorm else None
    kn = torch.rand(d, device=DEV) + 0.5 if qknorm else None
    kc = torch.zeros(nb, nkv, bs, d, device=DEV, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    kc2, vc2 = kc.clone().float(), vc.clone().float()
    qkv_ref = qkv.float().clone()
    got_q = ops.rope_and_cache(qkv.clone(), pos, cs, kc, vc, slots, nq, nkv, d, q_norm_w=qn, k_norm_w=kn,
                               rotary_dim=rd)
    from vllm_neuron_b200.ops import _ext

    import os
    os.environ["VLLM_B200_DISABLE_KERNELS"] = "1"
    try:
        want_q = ops.rope_and_cache(qkv_ref, pos, cs, kc2, vc2, slots, nq, nkv, d, q_norm_w=qn, k_norm_w=kn,
                                    rotary_dim=rd)
    finally:
        del os.environ["VLLM_B200_DISABLE_KERNELS"]
    _close(got_q, want_q, 3e-2, 2e-2, "q")
    _close(kc, kc2, 3e-2, 2e-2, "k cache")
    _close(vc, vc2, 1e-2, 1e-2, "v cache")


def _paged_setup(seq_lens, q_lens, nq, nkv, d, bs, dtype=torch.bfloat16, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    B = len(seq_lens)
    max_blocks = max(math.ceil(s / bs) for s in seq_lens) + 1
    nb = sum(math.ceil(s / bs) for s in seq_lens) + 4
    perm = torch.randperm(nb - 1, generator=g) + 1
    bt = torch.zeros(B, max_blocks, dtype=torch.int32)
    off = 0
    for i, s in enumerate(seq_lens):
        n = math.ceil(s / bs)
        bt[i, :n] = perm[off:off + n]
        off += n
    kc = (torch.randn(nb, nkv, bs, d, generator=g) * 1.0).to(DEV)
    vc = torch.randn(nb, nkv, bs, d, generator=g).to(DEV)
    T = sum(q_lens)
    q = torch.randn(T, nq, d, generator=g).to(DEV)
    qsl = torch.tensor([0] + list(torch.tensor(q_lens).cumsum(0)), dtype=torch.int32)
    return q, kc, vc, bt.to(DEV), torch.tensor(seq_lens, dtype=torch.int32, device=DEV), qsl.to(DEV)


@pytest.mark.parametrize("d", [64, 128, 256])
@pytest.mark.parametrize("window", [0, 128])
@pytest.mark.parametrize("splits", [1, 4, 5])  # 4: merged in a thread-block cluster; 5: workspace + combine
@pytest.mark.parametrize("fp8", [False, True])
@pytest.mark.parametrize("heads", [(16, 2), (12, 1), (4, 4)])  # GQA groups 8, 12 (rows 8..15 live), 1
def test_paged_decode(d, window, splits, fp8, heads):
    seq_lens = [1, 17, 100, 130, 1000, 3001]
    (nq, nkv), bs = heads, 32
    q, kc, vc, bt, sl, qsl = _paged_setup(seq_lens, [1] * len(seq_lens), nq, nkv, d, bs)
    sinks = torch.randn(nq, device=DEV)
    ks, vs = (0.05, 0.07) if fp8 else (1.0, 1.0)
    if fp8:
        kc8 = (kc / ks).to(torch.float8_e4m3fn)
        vc8 = (vc / vs).to(torch.float8_e4m3fn)
        kref, vref = kc8.float(), vc8.float()
        kk, vv = kc8, vc8
    else:
        kk, vv = kc.bfloat16(), vc.bfloat16()
        kref, vref = kk.float(), vv.float()
    qb = q.bfloat16()
    ws = torch.empty(len(seq_lens) * nq * splits * (d + 1), device=DEV)
    meta = AttentionMetadata(len(seq_lens), len(seq_lens), True, qsl, sl, bt, None, None, 1, max(seq_lens), ws,
                             splits)
    scale = d ** -0.5
    got = ops.attention(qb, kk, vv, meta, scale, sinks, window, ks, vs)
    want = ref.paged_attention(qb.float(), kref, vref, bt, sl, qsl, scale, sinks, window or None, ks, vs)
    _close(got, want, 2e-2, 3e-2, f"decode d={d} w={window} s={splits} fp8={fp8}")


@pytest.mark.parametrize("d", [64, 128, 256])
@pytest.mark.parametrize("window", [0, 128])
def test_paged_prefill(d, window):
    # chunked prefill / prefix hits: queries are the last q_len tokens of each sequence
    seq_lens = [70, 300, 129, 1000]
    q_lens = [70, 100, 1, 257]
    nq, nkv, bs = 8, 1, 16
    q, kc, vc, bt, sl, qsl = _paged_setup(seq_lens, q_lens, nq, nkv, d, bs, seed=3)
    sinks = torch.randn(nq, device=DEV)
    qb, kk, vv = q.bfloat16(), kc.bfloat16(), vc.bfloat16()
    meta = AttentionMetadata(sum(q_lens), len(seq_lens), False, qsl, sl, bt, None, None, max(q_lens), max(seq_lens))
    scale = d ** -0.5
    got = ops.attention(qb, kk, vv, meta, scale, sinks, window)
    want = ref.paged_attention(qb.float(), kk.float(), vv.float(), bt, sl, qsl, scale, sinks, window or None)
    _close(got, want, 2e-2, 3e-2, f"prefill d={d} w={window}")


@pytest.mark.parametrize("d", [64, 72, 128])
@pytest.mark.parametrize("causal", [True, False])
def test_varlen_attention(d, causal):
    torch.manual_seed(4)
    lens = [5, 64, 200, 130]
    T = sum(lens)
    nq, nkv = 4, 4
    q = torch.randn(T, nq, d, device=DEV, dtype=torch.bfloat16)
    k = torch.randn(T, nkv, d, device=DEV, dtype=torch.bfloat16)
    v = torch.randn(T, nkv, d, device=DEV, dtype=torch.bfloat16)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device=DEV)
    got = ops.varlen_attention(q, k, v, cu, d ** -0.5, causal, max(lens))
    want = ref.prefill_attention(q.float(), k.float(), v.float(), cu, d ** -0.5, None, None, causal)
    _close(got, want, 2e-2, 3e-2, f"varlen d={d}")


@pytest.mark.parametrize("T,E,H,k", [(64, 128, 2880, 4), (300, 128, 2880, 4), (16, 512, 2048, 10),
                                     (600, 128, 2880, 4), (1, 32, 2880, 4), (5, 64, 2048, 8), (40, 8, 256, 2)])
def test_router_topk_and_argmax(T, E, H, k):
    """GEMM (bf16 logits) + top-k softmax kernel: the chosen experts must be a top-k set of
    the fp32 reference logits up to bf16 rounding of the logits."""
    torch.manual_seed(5)
    x = torch.randn(T, H, device=DEV, dtype=torch.bfloat16)
    w = torch.randn(E, H, device=DEV, dtype=torch.bfloat16) * 0.02
    b = torch.randn(E, device=DEV, dtype=torch.bfloat16) * 0.02
    ids, wt = ops.router_topk(x, w, b, k)
    ref_logits = x.float() @ w.float().t() + b.float()
    kth = ref_logits.topk(k, -1).values[:, -1:]
    got = ref_logits.gather(1, ids.long())
    assert (got >= kth - 0.02).all(), "selected an expert outside the top-k"
    assert (ids.long().sort(-1).values.diff(dim=-1) > 0).all(), "duplicate expert"
    _close(wt, torch.softmax(got, -1), 1e-2, 1e-2, "router weights")
    # softmax over all experts, top-k, no renormalisation (Qwen3-Next without norm_topk_prob)
    ids_u, wt_u = ops.router_topk(x, w, b, k, "softmax_topk_unnormalized")
    assert torch.equal(ids_u, ids)
    _close(wt_u, torch.softmax(ref_logits, -1).gather(1, ids_u.long()), 1e-2, 1e-2, "unnormalised router weights")
    lg = torch.randn(64, 25136, device=DEV, dtype=torch.bfloat16)
    val, idx = ops.argmax(lg)
    assert torch.equal(idx, lg.float().argmax(-1))


def test_sampling():
    torch.manual_seed(6)
    B, V = 48, 50000
    logits = torch.randn(B, V, device=DEV) * 3
    temp = torch.rand(B, device=DEV) + 0.3
    temp[:4] = 0  # greedy rows
    topk = torch.randint(0, 300, (B,), device=DEV, dtype=torch.int32)
    topp = torch.rand(B, device=DEV) * 0.9 + 0.1
    u = torch.rand(B, device=DEV)
    got = ops.sample(logits, temp, topk, topp, u, 256)
    want = ref.sample(logits, temp, topk, topp, max_top_k=256, uniform=u)
    agree = (got == want).float().mean().item()
    assert agree >= 0.95, f"only {agree:.2%} of draws agree"
    assert torch.equal(got[:4], logits[:4].argmax(-1))


def _moe_reference(x, ids, wts, w13f, b13, w2f, b2, off, alpha, limit, emulate_fp8=True):
    """fp32 reference; with emulate_fp8 the activations go through the same MXFP8
    quantisation as the kernel (so the comparison isolates the GEMM)."""
    T, H = x.shape
    out = torch.zeros(T, H, device=x.device)
    E = w13f.shape[0]
    for e in range(E):
        tok, slot = torch.where(ids == e + off)
        if tok.numel() == 0:
            continue
        xe = x[tok].float()
        if emulate_fp8:
            xe = ref.dequant_mxfp8(*ref.quantize_mxfp8(xe))
        h = xe @ w13f[e].t() + b13[e]
        a = ref.clamped_swiglu(h[:, 0::2], h[:, 1::2], alpha, limit).bfloat16().float()
        if emulate_fp8:
            a = ref.dequant_mxfp8(*ref.quantize_mxfp8(a))
        y = (a @ w2f[e].t() + b2[e]) * wts[tok, slot][:, None]
        out.index_add_(0, tok, y.bfloat16().float())
    return out


@pytest.mark.parametrize("T,E,H,I,k,off,E_total,skew", [(16, 8, 256, 256, 2, 0, 8, 0), (39, 8, 256, 256, 2, 0, 8, 1),
                                                        (64, 32, 2880, 2880, 4, 0, 32, 0),
                                                        (200, 32, 2880, 2880, 4, 0, 32, 1),
                                                        (300, 16, 2880, 2880, 4, 16, 128, 0),
                                                        (1200, 8, 2880, 2880, 4, 0, 8, 1),
                                                        (4200, 8, 512, 512, 4, 0, 8, 1)])
def test_moe_mxfp4(T, E, H, I, k, off, E_total, skew):
    """skew=1 concentrates the routing so single experts get several N tiles."""
    from vllm_neuron_b200.ops.mx_layout import scales_to_atoms, tile_values

    g = torch.Generator(device=DEV).manual_seed(7)
    x = torch.randn(T, H, device=DEV, generator=g).bfloat16()
    w13 = torch.randint(0, 256, (E, 2 * I, H // 2), device=DEV, dtype=torch.uint8, generator=g)
    s13 = torch.randint(118, 123, (E, 2 * I, H // 32), device=DEV, dtype=torch.uint8, generator=g)
    w2 = torch.randint(0, 256, (E, H, I // 2), device=DEV, dtype=torch.uint8, generator=g)
    s2 = torch.randint(118, 123, (E, H, I // 32), device=DEV, dtype=torch.uint8, generator=g)
    b13 = torch.randn(E, 2 * I, device=DEV, generator=g) * 0.1
    b2 = torch.randn(E, H, device=DEV, generator=g) * 0.1
    logits = torch.randn(T, E_total, device=DEV, generator=g)
    if skew:
        logits[:, off] += 4.0
        logits[:, off + 1] += 3.0
    v, ids = torch.topk(logits, k, -1)
    wts = torch.softmax(v, -1)
    ids = ids.to(torch.int32)
    got = ops.moe_mxfp4(x, ids, wts, tile_values(w13, H), scales_to_atoms(s13, H), b13, tile_values(w2, I),
                        scales_to_atoms(s2, I), b2, off, 1.702, 7.0, H, I)
    w13f = ref.dequant_mxfp4(w13, s13)
    w2f = ref.dequant_mxfp4(w2, s2)
    want = _moe_reference(x, ids, wts, w13f, b13, w2f, b2, off, 1.702, 7.0)
    scale = want.abs().max().item()
    _close(got, want, 0.02 * scale, 0.03, f"moe T={T} E={E} H={H}")
    # and against unquantised bf16 activations (the model-level oracle), loosely
    want_bf16 = _moe_reference(x, ids, wts, w13f, b13, w2f, b2, off, 1.702, 7.0, emulate_fp8=False)
    rel = (got.float() - want_bf16).norm() / want_bf16.norm()
    assert rel < 0.08, f"relative error vs bf16 activations {rel:.3f}"
