"""Decode context parallelism: shard attention + LSE merge equals full attention (CPU
reference of the layout and merge), and a TP=2 / DCP=2 engine over gloo generates the same
greedy tokens as HF transformers."""

import pytest
import torch

from tiny_configs import workload
from vllm_neuron_b200 import ops
from vllm_neuron_b200.ops import reference as ref
from vllm_neuron_b200.ops.metadata import AttentionMetadata
from vllm_neuron_b200.parallel.dcp import merge_partials


def _layout(seq_lens, q_lens, hkv, d, bs, cp, seed=0):
    """A full cache of every sequence plus the per-rank DCP shards of the same tokens."""
    g = torch.Generator().manual_seed(seed)
    vbs = bs * cp
    nvb = [-(-L // vbs) for L in seq_lens]
    nb = sum(nvb) + 1
    bt = torch.zeros(len(seq_lens), max(nvb), dtype=torch.int32)
    perm = (torch.randperm(nb - 1, generator=g) + 1).tolist()
    off = 0
    for i, n in enumerate(nvb):
        bt[i, :n] = torch.tensor(perm[off:off + n])
        off += n
    # the full cache: token t of sequence i at block fb[i][t // bs]
    full_nb = sum(-(-L // bs) for L in seq_lens) + 1
    kf = torch.zeros(full_nb, hkv, bs, d)
    vf = torch.zeros(full_nb, hkv, bs, d)
    fbt = torch.zeros(len(seq_lens), max(-(-L // bs) for L in seq_lens), dtype=torch.int32)
    shards = [(torch.zeros(nb, hkv, bs, d), torch.zeros(nb, hkv, bs, d)) for _ in range(cp)]
    nxt = 1
    for i, L in enumerate(seq_lens):
        k = torch.randn(L, hkv, d, generator=g)
        v = torch.randn(L, hkv, d, generator=g)
        for t in range(L):
            if t % bs == 0:
                fbt[i, t // bs] = nxt
                nxt += 1
            kf[fbt[i, t // bs], :, t % bs] = k[t]
            vf[fbt[i, t // bs], :, t % bs] = v[t]
        pos = torch.arange(L)
        for r in range(cp):
            slots = ref.cp_slot_mapping(pos, bt, torch.full((L,), i), bs, r, cp)
            own = slots >= 0
            ref.write_kv_cache(k[own], v[own], shards[r][0], shards[r][1], slots[own])
    qsl = torch.tensor([0] + torch.tensor(q_lens).cumsum(0).tolist(), dtype=torch.int32)
    return kf, vf, fbt, shards, bt, torch.tensor(seq_lens, dtype=torch.int32), qsl


@pytest.mark.parametrize("cp", [2, 4])
@pytest.mark.parametrize("window", [0, 40])
@pytest.mark.parametrize("decode", [True, False])
def test_shards_merge_to_full_attention(cp, window, decode):
    torch.manual_seed(0)
    bs, hq, hkv, d = 8, 4, 2, 16
    seq_lens = [1, 9, 37, 100, 64]
    q_lens = [1] * 5 if decode else [1, 5, 20, 33, 64]
    kf, vf, fbt, shards, bt, sl, qsl = _layout(seq_lens, q_lens, hkv, d, bs, cp)
    T = sum(q_lens)
    q = torch.randn(T, hq, d)
    sinks = torch.randn(hq)
    scale = d ** -0.5
    want = ref.paged_attention(q, kf, vf, fbt, sl, qsl, scale, sinks, window or None)
    meta = AttentionMetadata(T, len(seq_lens), decode, qsl, sl, bt, None, None, max(q_lens), max(seq_lens))
    outs, lses = [], []
    for r in range(cp):
        o, lse = ops.attention_shard(q, shards[r][0], shards[r][1], meta, scale, window or None, 1.0, 1.0, r, cp)
        outs.append(o)
        lses.append(lse)
    lse_all = torch.stack(lses)
    got = sum(merge_partials(o, lse, lse_all, sinks) for o, lse in zip(outs, lses))
    torch.testing.assert_close(got, want.float(), rtol=1e-4, atol=1e-5)


def test_slot_mapping_deals_blocks_round_robin():
    bs, cp = 4, 2
    bt = torch.tensor([[7, 3]], dtype=torch.int32)
    pos = torch.arange(16)
    s0 = ref.cp_slot_mapping(pos, bt, torch.zeros(16, dtype=torch.long), bs, 0, cp).tolist()
    s1 = ref.cp_slot_mapping(pos, bt, torch.zeros(16, dtype=torch.long), bs, 1, cp).tolist()
    # tokens 0-3 and 8-11 on rank 0, 4-7 and 12-15 on rank 1; both ranks fill block 7 then 3
    assert s0 == [28, 29, 30, 31, -1, -1, -1, -1, 12, 13, 14, 15, -1, -1, -1, -1]
    assert s1 == [-1, -1, -1, -1, 28, 29, 30, 31, -1, -1, -1, -1, 12, 13, 14, 15]
    assert [ref.cp_count_local(x, bs, 0, cp) for x in (0, 3, 4, 8, 9, 13)] == [0, 3, 4, 4, 5, 8]
    assert [ref.cp_count_local(x, bs, 1, cp) for x in (0, 4, 5, 8, 12, 13)] == [0, 0, 1, 4, 4, 5]


def _hf_llama_one_kv_head():
    from transformers import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=2048, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=1, max_position_embeddings=1024,
                      rope_theta=10000.0, tie_word_embeddings=False)
    cfg._attn_implementation = "eager"
    return LlamaForCausalLM(cfg).eval().float(), cfg


def test_engine_dcp2_matches_hf(tmp_path, monkeypatch):
    from vllm_neuron_b200 import LLM, SamplingParams
    from vllm_neuron_b200.parallel import dcp
    from vllm_neuron_b200.utils.checkpoints import save_state_dict

    calls = {"n": 0}
    orig = dcp.dcp_attention

    def spy(*a, **k):
        calls["n"] += 1
        return orig(*a, **k)

    monkeypatch.setattr(dcp, "dcp_attention", spy)

    hf, cfg = _hf_llama_one_kv_head()
    d = cfg.to_dict()
    d["architectures"] = ["LlamaForCausalLM"]
    save_state_dict({k: v.detach().clone().contiguous() for k, v in hf.state_dict().items()}, str(tmp_path), d)
    prompts = workload(n=3, lo=30, hi=90, vocab=2048, seed=11)
    want = []
    with torch.no_grad():
        for p in prompts:
            g = hf.generate(torch.tensor([p]), max_new_tokens=12, do_sample=False, pad_token_id=0, eos_token_id=None)
            want.append(g[0, len(p):].tolist())
    # 48-token steps chunk the longer prompts, so prefill chunks also attend to the
    # context the other rank holds
    llm = LLM(model=str(tmp_path), dtype="float32", max_model_len=256, max_num_seqs=4, max_num_batched_tokens=48,
              block_size=8, device="cpu", tensor_parallel_size=2, decode_context_parallel_size=2, spmd=False)
    try:
        outs = llm.generate(prompt_token_ids=prompts,
                            sampling_params=SamplingParams(temperature=0, max_tokens=12, ignore_eos=True))
    finally:
        llm.shutdown()
    assert [o.outputs[0].token_ids for o in outs] == want
    assert calls["n"] > 0


@pytest.mark.gpu
@pytest.mark.parametrize("cp", [2, 4])
@pytest.mark.parametrize("window", [0, 100])
@pytest.mark.parametrize("mode", ["decode1", "decode4", "decode5", "prefill"])
def test_shard_kernels_merge_to_full_attention(cp, window, mode):
    """The paged decode / prefill kernels in shard mode (one GPU runs every rank's shard)."""
    torch.manual_seed(0)
    dev = "cuda"
    bs, hq, hkv, d = 32, 16, 2, 64
    seq_lens = [1, 40, 300, 1000, 2100]
    decode = mode != "prefill"
    q_lens = [1] * 5 if decode else [1, 40, 77, 130, 64]
    splits = {"decode1": 1, "decode4": 4, "decode5": 5, "prefill": 1}[mode]
    kf, vf, fbt, shards, bt, sl, qsl = _layout(seq_lens, q_lens, hkv, d, bs, cp, seed=3)
    T = sum(q_lens)
    q = torch.randn(T, hq, d).bfloat16()
    sinks = torch.randn(hq)
    scale = d ** -0.5
    want = ref.paged_attention(q.float(), kf.bfloat16().float(), vf.bfloat16().float(), fbt, sl, qsl, scale, sinks,
                               window or None)
    ws = torch.empty(T * hq * splits * (d + 1), device=dev)
    meta = AttentionMetadata(T, len(seq_lens), decode, qsl.to(dev), sl.to(dev), bt.to(dev), None, None,
                             max(q_lens), max(seq_lens), ws, splits)
    outs, lses = [], []
    for r in range(cp):
        o, lse = ops.attention_shard(q.to(dev), shards[r][0].bfloat16().to(dev), shards[r][1].bfloat16().to(dev),
                                     meta, scale, window or None, 1.0, 1.0, r, cp)
        outs.append(o)
        lses.append(lse)
    lse_all = torch.stack(lses)
    got = sum(merge_partials(o, lse, lse_all, sinks.to(dev)) for o, lse in zip(outs, lses)).cpu()
    torch.testing.assert_close(got, want.float(), rtol=2e-2, atol=2e-2)
