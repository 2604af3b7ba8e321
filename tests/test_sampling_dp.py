"""Sampling DP: batch <-> vocab all-to-all inside groups of TP ranks, one top-K per vocab
span, candidates gathered back.  Same tokens as the plain vocab-parallel sampler (TP=2 over
gloo, temperature / top-k / top-p sampling with host-supplied uniforms)."""

import torch

from tiny_configs import workload


def _ckpt(tmp_path):
    from transformers import LlamaConfig, LlamaForCausalLM

    from vllm_neuron_b200.utils.checkpoints import save_state_dict

    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=3000, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=512,
                      tie_word_embeddings=False)
    m = LlamaForCausalLM(cfg).eval().float()
    d = cfg.to_dict()
    d["architectures"] = ["LlamaForCausalLM"]
    save_state_dict({k: v.detach().clone().contiguous() for k, v in m.state_dict().items()}, str(tmp_path), d)
    return str(tmp_path)


def _run(path, sdp, monkeypatch=None):
    from vllm_neuron_b200 import LLM, SamplingParams

    calls = {"n": 0}
    if monkeypatch is not None:
        from vllm_neuron_b200.nn import sampler

        orig = sampler.Sampler._candidates_sdp

        def spy(self, *a, **k):
            calls["n"] += 1
            return orig(self, *a, **k)

        monkeypatch.setattr(sampler.Sampler, "_candidates_sdp", spy)
    llm = LLM(model=path, dtype="float32", max_model_len=256, max_num_seqs=8, max_num_batched_tokens=256,
              block_size=16, device="cpu", tensor_parallel_size=2, spmd=False, seed=7,
              additional_config={"neuron_config": {"on_device_sampling_config":
                                                   {"sampling_dp_degree": sdp, "max_top_k": 64}}})
    prompts = workload(n=5, lo=10, hi=40, vocab=3000, seed=3)
    try:
        outs = llm.generate(prompt_token_ids=prompts,
                            sampling_params=SamplingParams(temperature=0.9, top_k=40, top_p=0.9, max_tokens=12,
                                                           ignore_eos=True, seed=11))
    finally:
        llm.shutdown()
    return [o.outputs[0].token_ids for o in outs], calls["n"]


def test_sampling_dp_matches_vocab_parallel(tmp_path, monkeypatch):
    path = _ckpt(tmp_path)
    want, _ = _run(path, 1)
    got, n = _run(path, 2, monkeypatch)
    assert n > 0
    assert got == want
