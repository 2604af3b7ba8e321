"""Accuracy toolkit: two/three-way assertions, logit validation through the engine, tensor
capture and replacement hooks, KV-cache gathering (CPU)."""

import pytest
import torch

from test_llama_golden import _hf_llama, _save


def test_assert_close_two_and_three_way():
    from vllm_neuron_b200.accuracy import assert_close, assert_close_three_way

    torch.manual_seed(0)
    ref = torch.randn(64, 64)
    low = ref.bfloat16()
    assert_close(low, ref)
    with pytest.raises(AssertionError):
        assert_close(low + 0.5, ref)
    # kernel error comparable to the dtype's own error: passes
    r = assert_close_three_way(ref, low, (ref + 1e-3 * torch.randn_like(ref)).bfloat16())
    assert r.passed
    # an error well beyond bf16 rounding: target-specific
    with pytest.raises(AssertionError, match="target-specific"):
        assert_close_three_way(ref, low, (ref * 1.05).bfloat16())


@pytest.fixture(scope="module")
def llama(tmp_path_factory):
    m, cfg = _hf_llama()
    d = cfg.to_dict()
    d["architectures"] = ["LlamaForCausalLM"]
    path = tmp_path_factory.mktemp("acc")
    _save(m, d, path)
    return str(path), m


def test_logit_validation_through_engine(llama):
    from vllm_neuron_b200 import LLM
    from vllm_neuron_b200.accuracy import validate_greedy_generation, validate_prompt_logits

    path, hf = llama
    llm = LLM(model=path, dtype="float32", max_model_len=256, max_num_seqs=2, max_num_batched_tokens=128,
              block_size=16, device="cpu")
    try:
        prompts = [[5, 9, 100, 7, 3], list(range(20, 60))]
        checks = validate_greedy_generation(llm, hf, prompts, max_new_tokens=6)
        assert all(c.passed for c in checks), [c.gaps for c in checks]
        res = validate_prompt_logits(llm.engine, hf, prompts)
        assert all(r.top1_agree == 1.0 and r.max_abs < 1e-3 for r in res), res
    finally:
        llm.shutdown()


def test_tensor_capture_and_replacement(llama, tmp_path):
    from vllm_neuron_b200 import LLM, SamplingParams
    from vllm_neuron_b200.accuracy.tensor_capture import expand_patterns, load_captures

    assert expand_patterns(["layers.0-2.mlp"]) == ["layers.0.mlp", "layers.1.mlp", "layers.2.mlp"]
    path, _ = llama
    cap = str(tmp_path / "cap")
    nc = {"tensor_capture": {"modules": ["layers.0-1.self_attn"], "capture_dir": cap}}
    llm = LLM(model=path, dtype="float32", max_model_len=128, max_num_seqs=1, block_size=16, device="cpu",
              additional_config={"neuron_config": nc})
    out = llm.generate(prompt_token_ids=[[4, 5, 6, 7]], sampling_params=SamplingParams(temperature=0, max_tokens=3,
                                                                                        ignore_eos=True))
    llm.shutdown()
    caps = load_captures(cap)
    assert len(caps) == 3 and caps[0]["meta"]["kind"] == "prefill"
    assert caps[0]["tensors"]["layers.0.self_attn"].shape[0] == 4
    # replace layer 1's attention output with zeros at every step
    steps = [{"layers.1.self_attn": torch.zeros_like(c["tensors"]["layers.1.self_attn"])} for c in caps]
    llm2 = LLM(model=path, dtype="float32", max_model_len=128, max_num_seqs=1, block_size=16, device="cpu",
               additional_config={"neuron_config": {"tensor_replacement": {"tensors": steps}}})
    rep = llm2.engine.worker.runner.replacer
    out2 = llm2.generate(prompt_token_ids=[[4, 5, 6, 7]],
                         sampling_params=SamplingParams(temperature=0, max_tokens=3, ignore_eos=True))
    llm2.shutdown()
    assert rep.replaced == 3 and len(out2[0].outputs[0].token_ids) == 3


def test_kv_gather_matches_reference_write():
    from vllm_neuron_b200.accuracy.kv_cache_analysis import compare_kv, gather_request_kv
    from vllm_neuron_b200.ops import reference as ref

    torch.manual_seed(0)
    nb, H, bs, d, L = 6, 2, 4, 8, 10
    kc, vc = torch.zeros(nb, H, bs, d), torch.zeros(nb, H, bs, d)
    k, v = torch.randn(L, H, d), torch.randn(L, H, d)
    blocks = [3, 1, 5]
    slots = torch.tensor([blocks[p // bs] * bs + p % bs for p in range(L)])
    ref.write_kv_cache(k, v, kc, vc, slots)
    gk, gv = gather_request_kv(kc, vc, blocks, L)
    assert compare_kv(gk, k)["max_abs"] == 0 and compare_kv(gv, v)["first_bad_position"] is None


def test_tensor_compare_three_way_and_captures(tmp_path):
    import os

    from vllm_neuron_b200.accuracy.report import export_html, export_json
    from vllm_neuron_b200.accuracy.tensor_compare import (align_shapes, bhattacharyya, compare_captures,
                                                          compare_tensors, compare_tensors_three_way, report)
    from vllm_neuron_b200.accuracy.tensor_histogram import TensorHistogram, box_table

    torch.manual_seed(0)
    ref = torch.randn(64, 128)
    bf = ref.bfloat16().float()  # same-precision baseline
    good = ref.bfloat16().float() + 1e-4 * torch.randn_like(ref)
    bad = ref + 0.3 * torch.randn_like(ref)
    assert compare_tensors(good, ref, "good").passed and not compare_tensors(bad, ref, "bad").passed
    assert compare_tensors_three_way(good, bf, ref).passed and not compare_tensors_three_way(bad, bf, ref).passed
    assert bhattacharyya(ref, ref) > 0.999 and bhattacharyya(ref, ref + 100) < 0.01
    a, b = align_shapes(torch.zeros(1, 8, 4), torch.zeros(6, 4))  # padded capture vs real rows
    assert a.shape == b.shape == (6, 4)
    for d, t in (("a", good), ("b", ref)):
        os.makedirs(tmp_path / d)
        torch.save({"meta": {}, "tensors": {"layers.0": t, "norm": t * 2}}, tmp_path / d / "step_00000_rank0.pt")
    res, agg = compare_captures(str(tmp_path / "a"), str(tmp_path / "b"))
    assert agg.n == 2 and agg.n_failed == 0 and "2/2 passed" in report(res, agg)
    export_json(res, str(tmp_path / "r.json"))
    export_html(res, str(tmp_path / "r.html"))
    assert "<table>" in open(tmp_path / "r.html").read()
    h = TensorHistogram(torch.tensor([0.0, 1.0, 3.0, float("nan"), -0.25]), "x")
    assert h.nan == 1 and h.zeros == 1 and h.buckets == {-2: 1, 0: 1, 1: 1}
    assert "x" in h.render() and "p99" in box_table([h])
