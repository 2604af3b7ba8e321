"""EAGLE-3 speculative decoding on the GPU (bf16 target, random-init draft): every step
verifies the draft tokens with the target's multi-token pass (the prefill attention kernel
over the paged cache, the tcgen05 GEMMs), accepts the matching prefix and runs the draft's
catch-up and recurrent steps.  The greedy tokens are scored against the CPU fp32 engine on
the same checkpoint with teacher forcing: each must be the CPU argmax or within the bf16
logit-noise band of it.  Sampled generations with a fixed seed must repeat exactly."""

import pytest
import torch

from tiny_configs import workload

pytestmark = pytest.mark.gpu

DRAFT = {"architectures": ["Eagle3LlamaForCausalLM"], "hidden_size": 512, "num_attention_heads": 8,
         "num_key_value_heads": 2, "head_dim": 64, "intermediate_size": 1024, "vocab_size": 2048,
         "draft_vocab_size": 2048, "target_hidden_size": 512, "rms_norm_eps": 1e-5, "rope_theta": 10000.0}


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    from transformers import LlamaConfig, LlamaForCausalLM

    from vllm_neuron_b200.utils.checkpoints import save_state_dict

    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=2048, hidden_size=512, intermediate_size=1024, num_hidden_layers=4,
                      num_attention_heads=8, num_key_value_heads=2, max_position_embeddings=1024,
                      rope_theta=10000.0, tie_word_embeddings=False)
    m = LlamaForCausalLM(cfg).eval().float()
    d = cfg.to_dict()
    d["architectures"] = ["LlamaForCausalLM"]
    path = tmp_path_factory.mktemp("llama_spec")
    save_state_dict({k: v.detach().clone().contiguous() for k, v in m.state_dict().items()}, str(path), d)
    return str(path)


def _llm(path, device, dtype, spec):
    from vllm_neuron_b200 import LLM

    kw = dict(model=path, dtype=dtype, device=device, max_model_len=512, max_num_seqs=4,
              max_num_batched_tokens=256, block_size=32, seed=3)
    if spec:
        kw["speculative_config"] = {"num_speculative_tokens": 3, "draft_hf_config": dict(DRAFT)}
    return LLM(**kw)


def test_eagle3_greedy_on_gpu_matches_cpu_reference(ckpt):
    from vllm_neuron_b200 import SamplingParams
    from vllm_neuron_b200.accuracy.testing import greedy_logit_gaps

    prompts = workload(n=4, lo=20, hi=120, vocab=2048, seed=9)
    gpu = _llm(ckpt, "cuda", "bfloat16", True)
    try:
        outs = gpu.generate(prompt_token_ids=prompts,
                            sampling_params=SamplingParams(temperature=0, max_tokens=16, ignore_eos=True))
        gen = [list(o.outputs[0].token_ids) for o in outs]
        stats = dict(gpu.engine.proposer.stats)
    finally:
        gpu.shutdown()
    assert all(len(t) == 16 for t in gen)
    assert stats["proposed"] > 0 and stats["steps"] > 0, stats
    cpu = _llm(ckpt, "cpu", "float32", False)
    try:
        res = greedy_logit_gaps(cpu.engine, prompts, gen)
    finally:
        cpu.shutdown()
    assert res.outliers() <= res.n_tokens // 24, f"GPU speculative tokens far from the CPU argmax: {res}"
    assert res.exact_fraction >= 0.75, f"too few exact matches: {res}"


def test_eagle3_sampling_on_gpu_is_deterministic(ckpt):
    from vllm_neuron_b200 import SamplingParams

    prompts = workload(n=3, lo=20, hi=80, vocab=2048, seed=4)
    runs = []
    for _ in range(2):
        llm = _llm(ckpt, "cuda", "bfloat16", True)
        try:
            o = llm.generate(prompt_token_ids=prompts,
                             sampling_params=SamplingParams(temperature=0.8, top_k=40, max_tokens=12,
                                                            ignore_eos=True, seed=5))
            runs.append([list(x.outputs[0].token_ids) for x in o])
        finally:
            llm.shutdown()
    assert runs[0] == runs[1] and all(len(t) == 12 for t in runs[0])
