"""Llama (dense) and Qwen3 text decoders: greedy tokens vs HF transformers fp32 (CPU),
TP=1 and TP=2 over gloo."""

import pytest
import torch

from tiny_configs import workload


def _save(model, cfg_dict, path):
    from vllm_neuron_b200.utils.checkpoints import save_state_dict

    save_state_dict({k: v.detach().clone().contiguous() for k, v in model.state_dict().items()}, str(path), cfg_dict)


def _hf_llama():
    from transformers import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=2048, hidden_size=128, intermediate_size=256, num_hidden_layers=3,
                      num_attention_heads=8, num_key_value_heads=2, max_position_embeddings=1024,
                      rope_theta=500000.0, tie_word_embeddings=False,
                      rope_scaling={"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                                    "high_freq_factor": 4.0, "original_max_position_embeddings": 256})
    cfg._attn_implementation = "eager"
    return LlamaForCausalLM(cfg).eval().float(), cfg


def _hf_qwen3():
    from transformers import Qwen3Config, Qwen3ForCausalLM

    torch.manual_seed(0)
    cfg = Qwen3Config(vocab_size=2048, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=32, max_position_embeddings=1024,
                      rope_theta=1000000.0, tie_word_embeddings=True)
    cfg._attn_implementation = "eager"
    m = Qwen3ForCausalLM(cfg).eval().float()
    with torch.no_grad():
        for n, p in m.named_parameters():
            if "norm" in n:
                p.copy_(1 + 0.1 * torch.randn_like(p))
    return m, cfg


@pytest.fixture(scope="module", params=["llama", "qwen3"])
def ckpt(request, tmp_path_factory):
    m, cfg = _hf_llama() if request.param == "llama" else _hf_qwen3()
    d = cfg.to_dict()
    d["architectures"] = ["LlamaForCausalLM"]
    path = tmp_path_factory.mktemp(request.param)
    _save(m, d, path)
    return str(path), m


@pytest.mark.parametrize("tp", [1, 2])
def test_dense_greedy_matches_hf(ckpt, tp):
    from vllm_neuron_b200 import LLM, SamplingParams

    path, hf = ckpt
    prompts = workload(n=3, lo=20, hi=60, vocab=2048, seed=5)
    want = []
    with torch.no_grad():
        for p in prompts:
            g = hf.generate(torch.tensor([p]), max_new_tokens=10, do_sample=False, pad_token_id=0, eos_token_id=None)
            want.append(g[0, len(p):].tolist())
    llm = LLM(model=path, dtype="float32", max_model_len=256, max_num_seqs=4, max_num_batched_tokens=128,
              block_size=16, device="cpu", tensor_parallel_size=tp)
    try:
        outs = llm.generate(prompt_token_ids=prompts,
                            sampling_params=SamplingParams(temperature=0, max_tokens=10, ignore_eos=True))
    finally:
        llm.shutdown()
    assert [o.outputs[0].token_ids for o in outs] == want


def test_sequence_parallel_prefill_counts(ckpt, monkeypatch):
    """TP=2 prefill steps with an even token count run sequence-parallel layer boundaries
    (reduce-scatter + sharded residual + all-gather); greedy tokens still match HF."""
    from vllm_neuron_b200 import LLM, SamplingParams
    from vllm_neuron_b200.parallel import state as pstate

    calls = {"sp": 0}
    orig = pstate.GroupCoordinator._sp_add_rmsnorm

    def spy(self, *a, **k):
        calls["sp"] += 1
        return orig(self, *a, **k)

    monkeypatch.setattr(pstate.GroupCoordinator, "_sp_add_rmsnorm", spy)
    path, hf = ckpt
    prompts = [list(range(10, 40)), list(range(50, 70))]  # 50 tokens in one prefill step
    want = []
    with torch.no_grad():
        for p in prompts:
            g = hf.generate(torch.tensor([p]), max_new_tokens=4, do_sample=False, pad_token_id=0, eos_token_id=None)
            want.append(g[0, len(p):].tolist())
    llm = LLM(model=path, dtype="float32", max_model_len=256, max_num_seqs=4, max_num_batched_tokens=128,
              block_size=16, device="cpu", tensor_parallel_size=2, spmd=False,
              additional_config={"neuron_config": {"decode_batch_buckets": [2]}})
    try:
        outs = llm.generate(prompt_token_ids=prompts,
                            sampling_params=SamplingParams(temperature=0, max_tokens=4, ignore_eos=True))
    finally:
        llm.shutdown()
    assert [o.outputs[0].token_ids for o in outs] == want
    assert calls["sp"] > 0


def test_fp8_modelopt_checkpoint_close_to_dequantized_hf(tmp_path):
    """A static-FP8 (ModelOpt layout: e4m3 weights, per-tensor weight_scale and input_scale per
    projection; separate q / k / v and gate / up scales fused into per-row scales) checkpoint
    on the CPU path: logits close to HF fp32 with the dequantised weights (the remaining
    difference is the e4m3 rounding of the activations)."""
    from transformers import LlamaConfig, LlamaForCausalLM

    from vllm_neuron_b200 import LLM
    from vllm_neuron_b200.utils.checkpoints import save_state_dict

    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=2048, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                      num_attention_heads=8, num_key_value_heads=2, max_position_embeddings=1024,
                      tie_word_embeddings=False)
    m = LlamaForCausalLM(cfg).eval().float()
    sd, deq = {}, {}
    for k, v in m.state_dict().items():
        if k.endswith("proj.weight"):
            s = v.abs().amax() / 448 * (1.5 if "k_proj" in k or "up_proj" in k else 1.0)
            q = (v / s).clamp(-448, 448).to(torch.float8_e4m3fn)
            sd[k] = q
            sd[k.replace("weight", "weight_scale")] = s.reshape(())
            sd[k.replace("weight", "input_scale")] = torch.tensor(0.01)
            deq[k] = q.float() * s
        else:
            sd[k] = v.detach().clone().contiguous()
    m.load_state_dict({**m.state_dict(), **deq})
    d = cfg.to_dict()
    d["architectures"] = ["LlamaForCausalLM"]
    d["quantization_config"] = {"quant_method": "modelopt", "quant_algo": "FP8"}
    save_state_dict(sd, str(tmp_path), d)
    ids = torch.randint(1, 2000, (40,), generator=torch.Generator().manual_seed(1)).tolist()
    llm = LLM(model=str(tmp_path), dtype="float32", device="cpu", max_model_len=256, max_num_seqs=2,
              max_num_batched_tokens=128, block_size=16)
    try:
        got = llm.engine.score(ids).float()
    finally:
        llm.shutdown()
    with torch.no_grad():
        want = m(torch.tensor([ids])).logits[0].float()
    cos = torch.nn.functional.cosine_similarity(got, want, dim=-1)
    assert cos.min().item() > 0.99, cos.min().item()
