"""Qwen3-Next hybrid (gated DeltaNet + gated attention + shared-expert MoE): greedy tokens
vs HF transformers fp32 on CPU at TP=1 and TP=2 (gloo), including segmented prefill (the
recurrent state carried across prefill segments) and preemption-free concurrent decode."""

import pytest
import torch

from tiny_configs import hf_torch_path, workload

TINY = dict(vocab_size=2048, hidden_size=128, intermediate_size=256, num_hidden_layers=4, num_attention_heads=4,
            num_key_value_heads=2, head_dim=64, linear_conv_kernel_dim=4, linear_key_head_dim=32,
            linear_value_head_dim=32, linear_num_key_heads=4, linear_num_value_heads=8, num_experts=8,
            num_experts_per_tok=2, moe_intermediate_size=64, shared_expert_intermediate_size=64,
            max_position_embeddings=1024, tie_word_embeddings=False, rms_norm_eps=1e-6,
            rope_parameters={"rope_type": "default", "rope_theta": 10000.0, "partial_rotary_factor": 0.25})


def _hf():
    from transformers import Qwen3NextConfig, Qwen3NextForCausalLM

    torch.manual_seed(0)
    cfg = Qwen3NextConfig(**TINY)
    cfg._attn_implementation = "eager"
    m = Qwen3NextForCausalLM(cfg).eval().float()
    hf_torch_path(m)
    with torch.no_grad():
        for n, p in m.named_parameters():
            if "norm" in n or n.endswith("dt_bias"):
                p.copy_(0.1 * torch.randn_like(p) + (1.0 if n.endswith("linear_attn.norm.weight") else 0.0))
            elif "conv1d" in n:
                p.copy_(0.3 * torch.randn_like(p))
            elif n.endswith("A_log"):
                p.copy_(torch.log(torch.empty_like(p).uniform_(1, 16)))
    return m, cfg


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    from vllm_neuron_b200.utils.checkpoints import save_state_dict

    m, cfg = _hf()
    d = cfg.to_dict()
    d["architectures"] = ["Qwen3NextForCausalLM"]
    path = tmp_path_factory.mktemp("qwen3next")
    save_state_dict({k: v.detach().clone().contiguous() for k, v in m.state_dict().items()}, str(path), d)
    return str(path), m


@pytest.mark.parametrize("tp,chunk,dp,a2a", [(1, 256, 1, None), (1, 24, 1, None), (2, 256, 1, None),
                                             (1, 24, 2, None), (1, 24, 2, "naive"), (2, 256, 1, "naive")])
def test_qwen3_next_greedy_matches_hf(ckpt, tp, chunk, dp, a2a):
    from vllm_neuron_b200 import LLM, SamplingParams

    path, hf = ckpt
    prompts = workload(n=3, lo=20, hi=60, vocab=2048, seed=7)
    want = []
    with torch.no_grad():
        for p in prompts:
            g = hf.generate(torch.tensor([p]), max_new_tokens=8, do_sample=False, pad_token_id=0, eos_token_id=None)
            want.append(g[0, len(p):].tolist())
    llm = LLM(model=path, dtype="float32", max_model_len=256, max_num_seqs=4, max_num_batched_tokens=chunk,
              block_size=16, device="cpu", tensor_parallel_size=tp, data_parallel_size=dp,
              all2all_backend=a2a or "allgather_reducescatter", enable_expert_parallel=a2a is not None)
    try:
        outs = llm.generate(prompt_token_ids=prompts,
                            sampling_params=SamplingParams(temperature=0, max_tokens=8, ignore_eos=True))
        assert not llm.engine.worker.runner.slot_of  # every slot returned
    finally:
        llm.shutdown()
    assert [o.outputs[0].token_ids for o in outs] == want


def test_chunked_equals_recurrent_reference():
    """The chunked (WY / UT-transform) formulation used by the prefill kernel equals the
    token-by-token recurrence, including a carried-in state."""
    from vllm_neuron_b200.ops.reference import deltanet as dn

    torch.manual_seed(1)
    T, Hk, Hv, dk, dv = 150, 2, 4, 32, 16
    q, k = torch.randn(T, Hk, dk), torch.randn(T, Hk, dk)
    v = torch.randn(T, Hv, dv)
    g, beta = dn.gate_and_beta(torch.randn(T, Hv), torch.randn(T, Hv), torch.randn(Hv), torch.randn(Hv))
    s0 = torch.randn(2, Hv, dk, dv) * 0.1
    st_a, st_b = s0.clone(), s0.clone()
    qsl = torch.tensor([0, 70, 150])
    slots, init = torch.tensor([1, 0]), torch.tensor([1, 0])
    want = dn.gated_delta_rule(q, k, v, g, beta, st_a, qsl, slots, init)
    got = dn.chunked_gated_delta_rule(q, k, v, g, beta, st_b, qsl, slots, init, chunk=32)
    assert torch.allclose(got, want, atol=2e-4, rtol=1e-3), (got - want).abs().max()
    assert torch.allclose(st_b, st_a, atol=2e-4, rtol=1e-3)
