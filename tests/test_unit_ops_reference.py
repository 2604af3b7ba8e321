"""Reference-op semantics that the kernels are tested against."""

import torch

from vllm_neuron_b200.ops import reference as ref
from vllm_neuron_b200.ops.mx_layout import atoms_to_scales, pad_k, scales_to_atoms, tile_values, untile_values


def test_mxfp4_roundtrip_exact_on_grid():
    g = torch.Generator().manual_seed(0)
    codes = torch.randint(0, 256, (4, 64, 32), generator=g, dtype=torch.int32).to(torch.uint8)
    scales = torch.randint(110, 130, (4, 64, 2), generator=g, dtype=torch.int32).to(torch.uint8)
    w = ref.dequant_mxfp4(codes, scales)
    b2, s2 = ref.quantize_mxfp4(w)
    assert torch.equal(ref.dequant_mxfp4(b2, s2), w)


def test_mxfp8_error_bound():
    x = torch.randn(16, 256) * torch.logspace(-3, 3, 256)
    q, s = ref.quantize_mxfp8(x)
    y = ref.dequant_mxfp8(q, s)
    blk = x.view(16, 8, 32).abs().amax(-1, keepdim=True).expand(16, 8, 32).reshape(16, 256)
    assert ((y - x).abs() <= blk * 2 ** -3 + 1e-30).all()


def test_scale_atoms_roundtrip():
    s = torch.randint(0, 255, (2, 300, 90), dtype=torch.uint8)
    a = scales_to_atoms(s, 2880)
    assert a.shape == (2, 3, 23, 512)
    assert torch.equal(atoms_to_scales(a, 300, 2880), s)
    assert int(a.view(2, -1)[0, -1]) == 127  # padding never NaN
    assert pad_k(torch.ones(2, 3, 1440, dtype=torch.uint8), 2880).shape[-1] == 1472


def test_attention_sink_matches_concat_softmax():
    torch.manual_seed(0)
    q = torch.randn(5, 4, 16)
    k = torch.randn(5, 2, 16)
    v = torch.randn(5, 2, 16)
    sinks = torch.randn(4)
    cu = torch.tensor([0, 5])
    out = ref.prefill_attention(q, k, v, cu, 0.25, sinks, None)
    kk = k.repeat_interleave(2, 1)
    vv = v.repeat_interleave(2, 1)
    s = torch.einsum("qhd,khd->hqk", q, kk) * 0.25
    s = s.masked_fill(torch.triu(torch.ones(5, 5, dtype=torch.bool), 1), float("-inf"))
    full = torch.cat([s, sinks[:, None, None].expand(4, 5, 1)], -1).softmax(-1)[..., :-1]
    want = torch.einsum("hqk,khd->qhd", full, vv)
    assert torch.allclose(out, want, atol=1e-5)


def test_sliding_window_and_paged_equivalence():
    torch.manual_seed(1)
    L, H, d, bs = 40, 2, 8, 4
    q = torch.randn(L, H, d)
    k = torch.randn(L, H, d)
    v = torch.randn(L, H, d)
    dense = ref.prefill_attention(q, k, v, torch.tensor([0, L]), 0.3, None, 8)
    nb = L // bs + 1
    kc = torch.zeros(nb, H, bs, d)
    vc = torch.zeros(nb, H, bs, d)
    slots = torch.arange(L) + bs  # blocks 1..
    ref.write_kv_cache(k, v, kc, vc, slots)
    bt = torch.arange(1, nb)[None].int()
    paged = ref.paged_attention(q[-7:], kc, vc, bt, torch.tensor([L]), torch.tensor([0, 7]), 0.3, None, 8)
    assert torch.allclose(paged, dense[-7:], atol=1e-5)


def test_lse_merge_equals_full():
    torch.manual_seed(2)
    q = torch.randn(3, 2, 8)
    k = torch.randn(20, 2, 8)
    v = torch.randn(20, 2, 8)
    sinks = torch.randn(2)
    qp = torch.arange(17, 20)
    full, _ = ref.attention._attend(q, k, v, qp, torch.arange(20), 0.5, sinks, None)
    o1, l1 = ref.attention._attend(q, k[:9], v[:9], qp, torch.arange(9), 0.5, None, None)
    o2, l2 = ref.attention._attend(q, k[9:], v[9:], qp, torch.arange(9, 20), 0.5, None, None)
    merged = ref.lse_merge([o1, o2], [l1, l2], sinks)
    assert torch.allclose(merged, full, atol=1e-5)


def test_router_and_moe_reference():
    torch.manual_seed(3)
    x = torch.randn(6, 32)
    w = torch.randn(8, 32)
    ids, wt, logits = ref.router_topk(x, w, None, 2)
    assert torch.allclose(wt.sum(-1), torch.ones(6))
    assert torch.equal(ids.long(), logits.topk(2, -1).indices)
    w13 = torch.randn(8, 16, 32) * 0.1
    w2 = torch.randn(8, 32, 8) * 0.1
    full = ref.moe_experts(x, ids, wt, w13, None, w2, None)
    part = ref.moe_experts(x, ids, wt, w13[:4], None, w2[:4], None, expert_offset=0) + \
        ref.moe_experts(x, ids, wt, w13[4:], None, w2[4:], None, expert_offset=4)
    assert torch.allclose(full, part, atol=1e-5)  # expert-parallel partial sums add up


def test_blockwise_mapping_and_topk_reduce():
    ids = torch.tensor([[0, 2], [2, 1], [0, 1]], dtype=torch.int32)
    tp, b2e, offs = ref.build_blockwise_mapping(ids, 3, 2)
    assert b2e.tolist() == [0, 1, 2] and offs.tolist() == [0, 1, 2, 3]
    assert sorted(tp[:2].tolist()) == [0, 4]
    rows = torch.arange(12.0).view(4, 3)
    out = ref.topk_reduce(rows, torch.tensor([1, 2, 1, 0]), 2)
    assert out.tolist() == [[6.0, 8.0, 10.0], [3.0, 4.0, 5.0]]


def test_sampling_reference():
    torch.manual_seed(4)
    logits = torch.randn(4, 100)
    t = torch.tensor([0.0, 1.0, 0.5, 2.0])
    out = ref.sample(logits, t, torch.tensor([0, 1, 5, 0]), torch.tensor([1.0, 1.0, 0.5, 1.0]),
                     uniform=torch.tensor([0.3, 0.9, 0.1, 0.999]))
    assert out[0] == logits[0].argmax() and out[1] == logits[1].argmax()  # greedy and top_k=1
    top5 = logits[2].topk(5).indices
    assert out[2] in top5


def test_rejection_and_spec_correction():
    drafts = torch.tensor([[1, 2, 3], [1, 9, 3]])
    target = torch.tensor([[1, 2, 3, 4], [1, 2, 3, 4]])
    out = ref.rejection_greedy(drafts, target)
    assert out.tolist() == [[1, 2, 3, 4], [1, 2, -1, -1]]
    pos, slots = ref.correct_spec_decode_positions_and_slot_mapping(
        torch.tensor([[10, 11]]), torch.tensor([[0, 0]]), torch.tensor([2]), torch.tensor([[5, 6, 7]]), 4)
    assert pos.tolist() == [[8, 9]] and slots.tolist() == [[7 * 4 + 0, 7 * 4 + 1]]  # block_tables[0][8 // 4] = 7


def test_yarn_matches_hf():
    from transformers import GptOssConfig
    from transformers.modeling_rope_utils import ROPE_INIT_FUNCTIONS

    cfg = GptOssConfig(head_dim=64)
    inv_hf, af_hf = ROPE_INIT_FUNCTIONS["yarn"](cfg, "cpu")
    inv, af = ref.yarn_inv_freq(64, 150000.0, 32.0, 4096, 32.0, 1.0, False)
    assert torch.allclose(inv, inv_hf.float(), rtol=1e-5) and abs(af - af_hf) < 1e-6


def test_value_tiles_roundtrip():
    v = torch.randint(0, 255, (2, 300, 1440), dtype=torch.uint8)
    t = tile_values(v, 2880)
    assert t.shape == (2, 3, 23, 128, 64)
    assert torch.equal(untile_values(t, 300, 2880), v)
    assert torch.equal(t[1, 2, 5, 10], v[1, 266, 320:384])  # row 2*128+10, K bytes 5*64..


def test_mla_decode_reference_matches_naive_loop():
    """The MLA decode reference (paged latent cache shared by every head) against an explicit
    per-head, per-token computation; the CPU wrapper routes to it."""
    import math

    from vllm_neuron_b200 import ops
    from vllm_neuron_b200.ops.reference.attention import mla_decode

    g = torch.Generator().manual_seed(3)
    B, Hq, bs, lens = 2, 4, 4, [5, 9]
    cache = torch.randn(8, bs, 576, generator=g)
    bt = torch.tensor([[3, 1, 0], [7, 2, 5]], dtype=torch.int32)
    q = torch.randn(B, Hq, 576, generator=g)
    sl = torch.tensor(lens, dtype=torch.int32)
    got = mla_decode(q, cache, bt, sl, 0.07)
    for b in range(B):
        rows = [cache[int(bt[b, t // bs]), t % bs] for t in range(lens[b])]
        for h in range(Hq):
            s = [0.07 * float(q[b, h] @ r) for r in rows]
            m = max(s)
            w = [math.exp(x - m) for x in s]
            o = sum(wi * r[:512] for wi, r in zip(w, rows)) / sum(w)
            assert torch.allclose(got[b, h], o, atol=1e-5)
    assert torch.allclose(ops.mla_decode(q, cache, bt, sl, 0.07), got)
