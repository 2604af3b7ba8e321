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
