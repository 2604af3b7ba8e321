"""EAGLE-3 speculative decoding: greedy output with speculation must equal greedy output
without it (verification accepts only tokens the target would have produced)."""

import pytest
import torch

from tiny_configs import workload

TARGET = {"architectures": ["LlamaForCausalLM"], "model_type": "llama", "vocab_size": 2048, "hidden_size": 128,
          "intermediate_size": 256, "num_hidden_layers": 6, "num_attention_heads": 8, "num_key_value_heads": 2,
          "max_position_embeddings": 1024, "rope_theta": 10000.0, "rms_norm_eps": 1e-5}
DRAFT = {"architectures": ["Eagle3LlamaForCausalLM"], "hidden_size": 128, "num_attention_heads": 4,
         "num_key_value_heads": 2, "head_dim": 32, "intermediate_size": 256, "vocab_size": 2048,
         "draft_vocab_size": 2048, "target_hidden_size": 128, "rms_norm_eps": 1e-5, "rope_theta": 10000.0}


def _run(spec):
    from vllm_neuron_b200 import LLM, SamplingParams

    kw = dict(hf_config=dict(TARGET), load_format="dummy", dtype="float32", max_model_len=256, max_num_seqs=4,
              max_num_batched_tokens=128, block_size=16, device="cpu", seed=3)
    if spec:
        kw["speculative_config"] = {"num_speculative_tokens": 3, "draft_hf_config": dict(DRAFT)}
    llm = LLM(**kw)
    prompts = workload(n=3, lo=10, hi=40, vocab=2048, seed=9)
    outs = llm.generate(prompt_token_ids=prompts,
                        sampling_params=SamplingParams(temperature=0, max_tokens=12, ignore_eos=True))
    stats = llm.engine.proposer.stats if spec else None
    llm.shutdown()
    return [o.outputs[0].token_ids for o in outs], stats


def test_eagle3_greedy_is_lossless():
    base, _ = _run(False)
    spec, stats = _run(True)
    assert spec == base
    assert stats["proposed"] > 0 and stats["steps"] > 0


def test_rejection_sampling_preserves_distribution():
    """With a one-hot (greedy) draft, the first emitted token of rejection sampling is
    distributed as the target sampling distribution p (temperature / top-k / top-p)."""
    from vllm_neuron_b200.ops import reference as ref
    from vllm_neuron_b200.spec_decode.rejection_sampler import rejection_sample

    torch.manual_seed(0)
    V, N = 12, 40000
    logits = torch.randn(V) * 1.5
    cand_v = logits[None].expand(N, V).contiguous()
    cand_i = torch.arange(V)[None].expand(N, V).contiguous()
    temp = torch.full((N,), 0.8)
    topk = torch.full((N,), 8, dtype=torch.int32)
    topp = torch.full((N,), 0.95)
    draft = torch.full((N,), int(logits.argsort()[-2]), dtype=torch.int64)  # a likely but not top token
    tok, acc = rejection_sample(cand_v, cand_i, draft, temp, topk, topp, torch.rand(N), torch.rand(N))
    probs, ids = ref.topk_topp_filter(logits[None] / 0.8, topk[:1], topp[:1])
    p = torch.zeros(V)
    p[ids[0]] = probs[0]
    emp = torch.bincount(tok, minlength=V).float() / N
    assert (emp - p).abs().max() < 0.012, (emp, p)
    assert abs(acc.float().mean().item() - p[draft[0]].item()) < 0.012
    # greedy rows: accept iff the draft is the argmax, else emit the argmax
    temp0 = torch.zeros(N)
    tok0, acc0 = rejection_sample(cand_v, cand_i, draft, temp0, topk, topp, torch.rand(N), torch.rand(N))
    assert not acc0.any() and (tok0 == int(logits.argmax())).all()


def test_eagle3_with_sampling_runs_and_is_deterministic():
    from vllm_neuron_b200 import LLM, SamplingParams

    outs = []
    for _ in range(2):
        kw = dict(hf_config=dict(TARGET), load_format="dummy", dtype="float32", max_model_len=256, max_num_seqs=4,
                  max_num_batched_tokens=128, block_size=16, device="cpu", seed=3,
                  speculative_config={"num_speculative_tokens": 3, "draft_hf_config": dict(DRAFT)})
        llm = LLM(**kw)
        prompts = workload(n=3, lo=10, hi=40, vocab=2048, seed=9)
        o = llm.generate(prompt_token_ids=prompts,
                         sampling_params=SamplingParams(temperature=0.9, top_k=50, max_tokens=12, ignore_eos=True,
                                                        seed=5))
        outs.append([x.outputs[0].token_ids for x in o])
        llm.shutdown()
    assert outs[0] == outs[1] and all(len(t) == 12 for t in outs[0])
