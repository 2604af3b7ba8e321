"""The tensor-core prefill attention (``csrc/fa_prefill.cu``: tcgen05 MMAs with S and O in
TMEM, K/V tiles by TMA from the paged cache) against the fp32 PyTorch reference of the same
op: fresh prompts and chunked prefill over a cached prefix, sinks, a sliding window, GQA,
block sizes 16 and 32, queries read from the fused QKV projection (row stride > heads x d)."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _setup(seq_lens, q_lens, nq, nkv, bs, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    d = 64
    B = len(seq_lens)
    max_blocks = max(math.ceil(s / bs) for s in seq_lens) + 2
    nb = sum(math.ceil(s / bs) for s in seq_lens) + 3
    perm = torch.randperm(nb - 1, generator=g) + 1
    bt = torch.zeros(B, max_blocks, dtype=torch.int32)
    off = 0
    for i, s in enumerate(seq_lens):
        n = math.ceil(s / bs)
        bt[i, :n] = perm[off:off + n]
        off += n
    kc = torch.randn(nb, nkv, bs, d, generator=g).bfloat16().to(DEV)
    vc = torch.randn(nb, nkv, bs, d, generator=g).bfloat16().to(DEV)
    T = sum(q_lens)
    # queries as the q part of a fused [T, (nq + 2 nkv) d] projection
    qkv = torch.randn(T, (nq + 2 * nkv) * d, generator=g).bfloat16().to(DEV)
    q = qkv[:, : nq * d].view(T, nq, d)
    qsl = torch.tensor([0] + list(torch.tensor(q_lens).cumsum(0)), dtype=torch.int32, device=DEV)
    return q, kc, vc, bt.to(DEV), torch.tensor(seq_lens, dtype=torch.int32, device=DEV), qsl


@pytest.mark.parametrize("bs", [16, 32])
@pytest.mark.parametrize("window", [0, 128])
@pytest.mark.parametrize("heads", [(8, 1), (16, 2), (4, 4)])
def test_tc_prefill_matches_reference(bs, window, heads):
    from vllm_neuron_b200 import ops
    from vllm_neuron_b200.ops import reference as ref
    from vllm_neuron_b200.ops.metadata import AttentionMetadata

    nq, nkv = heads
    seq_lens = [700, 70, 300, 129, 1000, 2048]
    q_lens = [700, 70, 100, 1, 257, 512]  # fresh prompts and chunks after a cached prefix
    q, kc, vc, bt, sl, qsl = _setup(seq_lens, q_lens, nq, nkv, bs, seed=bs + window + nq)
    sinks = torch.randn(nq, device=DEV)
    meta = AttentionMetadata(sum(q_lens), len(seq_lens), False, qsl, sl, bt, None, None, max(q_lens),
                             max(seq_lens))
    scale = 64 ** -0.5
    got = ops.attention(q, kc, vc, meta, scale, sinks, window)
    torch.cuda.synchronize()
    want = ref.paged_attention(q.float(), kc.float(), vc.float(), bt, sl, qsl, scale, sinks, window or None)
    err = (got.float() - want).abs()
    tol = 2e-2 + 3e-2 * want.abs()
    bad = (err > tol).sum().item()
    assert bad == 0, f"{bad} mismatches, max err {err.max().item():.4g}"
    assert ops.check_device_status(q.device) == 0


def test_tc_prefill_without_sinks_and_exact_tile_edges():
    """Query and key counts on 128 boundaries (full tiles only) and a sequence whose window
    starts inside a tile; no sinks."""
    from vllm_neuron_b200 import ops
    from vllm_neuron_b200.ops import reference as ref
    from vllm_neuron_b200.ops.metadata import AttentionMetadata

    seq_lens, q_lens = [256, 384, 640], [128, 384, 256]
    q, kc, vc, bt, sl, qsl = _setup(seq_lens, q_lens, 8, 2, 32, seed=11)
    meta = AttentionMetadata(sum(q_lens), 3, False, qsl, sl, bt, None, None, max(q_lens), max(seq_lens))
    for window in (0, 200):
        got = ops.attention(q, kc, vc, meta, 0.125, None, window)
        want = ref.paged_attention(q.float(), kc.float(), vc.float(), bt, sl, qsl, 0.125, None, window or None)
        err = (got.float() - want).abs()
        assert (err > 2e-2 + 3e-2 * want.abs()).sum().item() == 0, f"window {window}: max err {err.max().item()}"


@pytest.mark.parametrize("window", [0, 128])
def test_mixed_step_attention_matches_reference(window):
    """A mixed step: single-token decode sequences first (decode kernel on their rows), then
    prompt chunks (tensor-core prefill kernel), in one ops.attention call."""
    from vllm_neuron_b200 import ops
    from vllm_neuron_b200.ops import reference as ref
    from vllm_neuron_b200.ops.metadata import AttentionMetadata

    seq_lens = [300, 1500, 77, 1024, 640, 200]
    q_lens = [1, 1, 1, 1, 256, 200]
    q, kc, vc, bt, sl, qsl = _setup(seq_lens, q_lens, 8, 1, 32, seed=21 + window)
    sinks = torch.randn(8, device=DEV)
    splits = 4
    ws = torch.empty(len(seq_lens) * 8 * splits * 65, device=DEV)
    meta = AttentionMetadata(sum(q_lens), len(seq_lens), False, qsl, sl, bt, None, None, max(q_lens),
                             max(seq_lens), workspace=ws, num_splits=splits, num_decode_seqs=4)
    got = ops.attention(q, kc, vc, meta, 0.125, sinks, window)
    torch.cuda.synchronize()
    want = ref.paged_attention(q.float(), kc.float(), vc.float(), bt, sl, qsl, 0.125, sinks, window or None)
    err = (got.float() - want).abs()
    assert (err > 2e-2 + 3e-2 * want.abs()).sum().item() == 0, f"max err {err.max().item()}"
    assert ops.check_device_status(q.device) == 0
