"""Component DP (embedding / lm_head / mlp sharded over TP x DP supergroups, rows gathered
over the DP replicas and sliced back): DP=2 replicas over gloo give HF's greedy tokens and the
same sampled tokens as plain DP."""

import torch

from tiny_configs import workload


def _ckpt(tmp_path):
    from transformers import LlamaConfig, LlamaForCausalLM

    from vllm_neuron_b200.utils.checkpoints import save_state_dict

    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=2001, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=512,
                      tie_word_embeddings=False)
    cfg._attn_implementation = "eager"
    m = LlamaForCausalLM(cfg).eval().float()
    d = cfg.to_dict()
    d["architectures"] = ["LlamaForCausalLM"]
    save_state_dict({k: v.detach().clone().contiguous() for k, v in m.state_dict().items()}, str(tmp_path), d)
    return str(tmp_path), m


def _run(path, comp: bool, sp, monkeypatch=None):
    from vllm_neuron_b200 import LLM

    calls = {"n": 0}
    if monkeypatch is not None:
        from vllm_neuron_b200.engine import model_runner

        orig = model_runner.ModelRunner._sample_lm_dp

        def spy(self, *a, **k):
            calls["n"] += 1
            return orig(self, *a, **k)

        monkeypatch.setattr(model_runner.ModelRunner, "_sample_lm_dp", spy)
    nc = {"embedding_dp_size": 2, "lm_head_dp_size": 2, "mlp_dp_size": 2} if comp else {}
    llm = LLM(model=path, dtype="float32", max_model_len=256, max_num_seqs=4, max_num_batched_tokens=128,
              block_size=16, device="cpu", data_parallel_size=2, additional_config={"neuron_config": nc})
    prompts = workload(n=5, lo=10, hi=50, vocab=2001, seed=9)
    try:
        outs = llm.generate(prompt_token_ids=prompts, sampling_params=sp)
    finally:
        llm.shutdown()
    return prompts, [o.outputs[0].token_ids for o in outs], calls["n"]


def test_component_dp_greedy_matches_hf(tmp_path, monkeypatch):
    from vllm_neuron_b200 import SamplingParams

    path, hf = _ckpt(tmp_path)
    prompts, got, n = _run(path, True, SamplingParams(temperature=0, max_tokens=8, ignore_eos=True), monkeypatch)
    want = []
    with torch.no_grad():
        for p in prompts:
            g = hf.generate(torch.tensor([p]), max_new_tokens=8, do_sample=False, pad_token_id=0, eos_token_id=None)
            want.append(g[0, len(p):].tolist())
    assert n > 0
    assert got == want


def test_component_dp_sampling_matches_plain_dp(tmp_path):
    from vllm_neuron_b200 import SamplingParams

    path, _ = _ckpt(tmp_path)
    sp = SamplingParams(temperature=0.8, top_k=30, top_p=0.95, max_tokens=8, ignore_eos=True, seed=5)
    _, want, _ = _run(path, False, sp)
    _, got, _ = _run(path, True, sp)
    assert got == want
