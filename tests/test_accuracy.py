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


def _hf_greedy_fn(hf, n_new):
    """generate_fn over an HF model: greedy continuation of every sequence, logits [n, B, V]."""
    base = {}

    def fn(ids):
        base.setdefault("n", len(ids[0]))
        n = n_new - (len(ids[0]) - base["n"])
        rows = []
        with torch.no_grad():
            for x in ids:
                seq, out = list(x), []
                for _ in range(n):
                    lg = hf(torch.tensor([seq])).logits[0, -1].float()
                    out.append(lg)
                    seq.append(int(lg.argmax()))
                rows.append(torch.stack(out))
        return torch.stack(rows, 1)

    return fn


def test_debug_logits_dump_matches_hf(llama, tmp_path):
    """neuron_config.debug_logits_dir: one file per sampling step; rows at positions
    prompt_len - 1 ... carry the decode path's full-vocab logits (chunked prefill writes no
    partial-chunk rows), equal to the HF model's teacher-forced logits."""
    from vllm_neuron_b200 import LLM, SamplingParams
    from vllm_neuron_b200.engine.debug_logits import read_debug_logits, stack_debug_logits

    path, hf = llama
    d = str(tmp_path / "logits")
    llm = LLM(model=path, dtype="float32", max_model_len=256, max_num_seqs=2, max_num_batched_tokens=16,
              block_size=16, device="cpu", additional_config={"neuron_config": {"debug_logits_dir": d}})
    try:
        prompts = [[5, 9, 100, 7, 3], list(range(20, 45))]  # the second prefills in two chunks
        outs = llm.generate(prompt_token_ids=prompts,
                            sampling_params=SamplingParams(temperature=0, max_tokens=4, ignore_eos=True))
    finally:
        llm.shutdown()
    got = read_debug_logits(d)
    assert [sorted(v) for _, v in sorted(got.items())] == [[4, 5, 6, 7], [24, 25, 26, 27]]
    lg = stack_debug_logits(d)
    assert lg.shape[:2] == (4, 2)
    for b, (p, o) in enumerate(zip(prompts, outs)):
        toks = list(o.outputs[0].token_ids)
        assert lg[:, b].argmax(-1).tolist() == toks
        with torch.no_grad():
            want = hf(torch.tensor([p + toks])).logits[0, len(p) - 1:len(p) + 3].float()
        assert torch.allclose(lg[:, b], want, atol=1e-4), (lg[:, b] - want).abs().max()


def test_logit_validation_tiers_divergence_three_way():
    """Teacher-forced validator on synthetic logits: identical logits pass; a constant offset is
    removed; noise beyond the top-5 tier fails; a flipped near-tie within one bf16 ULP passes
    and is re-prompted with the teacher token; three-way metrics against fp32 logits."""
    from vllm_neuron_b200.accuracy.logit_validation import check_token_logits, logit_validation, ulp

    assert ulp(19.0) == 0.125 and ulp(1.0, 23) == 2.0 ** -23
    torch.manual_seed(0)
    S, B, V = 6, 2, 64
    exp = torch.randn(S, B, V) * 4
    calls = []

    def fn_from(actual):
        def fn(ids):
            done = len(ids[0]) - 3
            calls.append(done)
            return actual[done:]
        return fn

    ids = [[1, 2, 3], [4, 5, 6]]
    assert logit_validation(ids, fn_from(exp.clone()), exp).passed
    assert ids == [[1, 2, 3], [4, 5, 6]]  # caller's lists untouched
    assert logit_validation(ids, fn_from(exp + 2.5), exp).passed  # constant offset removed
    noisy = exp.clone()
    top = exp[3, 1].topk(2).indices
    noisy[3, 1, top[1]] -= 0.5  # the second-best entry off by 0.5 / max|e| ~ 5%: over the top-5 tier
    r = logit_validation(ids, fn_from(noisy), exp)
    assert not r.passed and [(t.batch, t.index) for t in r.failures()] == [(1, 3)]
    # a near-tie flipped by less than one bf16 ULP: divergent but in bounds
    tie = exp.clone()
    w = exp[2, 0].argmax()
    other = (w + 1) % V
    tie[2, 0, other] = tie[2, 0, w] + ulp(float(tie[2, 0, w])) / 4
    exp2 = tie.clone()
    exp2[2, 0, other] = tie[2, 0, w] - ulp(float(tie[2, 0, w])) / 4
    calls.clear()
    r = logit_validation(ids, fn_from(tie), exp2)
    assert r.passed and sum(t.divergence for t in r.tokens[0]) == 1
    assert calls == [0, 3]  # re-prompted after the divergent position
    # a flip by many ULPs fails
    far = exp.clone()
    far[2, 0, other] = far[2, 0, w] + 1.0
    assert not logit_validation(ids, fn_from(far), exp).passed
    # three-way: target error like the expected tensor's own error vs fp32 -> metrics pass
    fp32 = exp.clone()
    low = fp32.bfloat16().float()
    tgt = (fp32 + 1e-3 * torch.randn_like(fp32)).bfloat16().float()
    r = logit_validation(ids, fn_from(tgt), low, baseline_logits=fp32)
    tw = [t.three_way for row in r.tokens for t in row]
    assert all(m is not None for m in tw) and sum(m["passed"] for m in tw) >= len(tw) // 2
    c = check_token_logits(exp[0, 0], exp[0, 0], actual_token=int(exp[0, 0].argmax()))
    assert c.passed and not c.divergence and c.shift == pytest.approx(0.0, abs=1e-5)


def test_multi_prompt_and_engine_generate_fn(llama, tmp_path):
    """Engine (real decode path via its logit dumps) against HF fp32 with teacher forcing,
    over two prompts, with HF in float64 as the three-way baseline; and one prompt replicated
    to a batch of three."""
    import copy

    from vllm_neuron_b200 import LLM
    from vllm_neuron_b200.accuracy import make_engine_generate_fn, multi_prompt_logit_validation

    path, hf = llama
    hf64 = copy.deepcopy(hf).double()
    d = str(tmp_path / "dbg")
    llm = LLM(model=path, dtype="float32", max_model_len=256, max_num_seqs=4, max_num_batched_tokens=64,
              block_size=16, device="cpu", additional_config={"neuron_config": {"debug_logits_dir": d}})
    try:
        prompts = [[[5, 9, 100, 7, 3]], [list(range(30, 50)), list(range(60, 70))]]
        expected = [_hf_greedy_fn(hf, 5)(p) for p in prompts]
        fp64 = [_hf_greedy_fn(hf64, 5)(p).float() for p in prompts]
        for p, e in zip(prompts, expected):  # engine vs HF fp32: two-way
            r = multi_prompt_logit_validation([p], make_engine_generate_fn(llm, 5, d), [e])
            assert r.passed, r.per_prompt[0].summary()
        r = multi_prompt_logit_validation(prompts, make_engine_generate_fn(llm, 5, d), expected,
                                          prompts_baseline_logits=fp64)
        assert r.passed, [x.summary() for x in r.per_prompt]
        agg = r.aggregate
        assert set(agg) >= {"pp_static_0.03", "pp_max_linf_1.5x", "agg_bc", "agg_sigma_ratio", "per_token_bc"}
        assert len(agg["per_token_bc"]) == 5 and 0 < agg["agg_sigma_ratio"] < float("inf")
        rep = multi_prompt_logit_validation([prompts[0]], make_engine_generate_fn(llm, 5, d), [expected[0]],
                                            replicate_to_batch_size=3)
        assert rep.passed and len(rep.per_prompt[0].tokens) == 3
    finally:
        llm.shutdown()



def test_kv_snapshot_matches_hf_cache(llama):
    """The engine's KV of a finished request (snapshot taken before its blocks are freed)
    equals the HF model's cache on prompt + output[:-1]; three-way against HF float64 with
    per-layer error-distribution overlap and the cross-prompt aggregates."""
    import copy

    from vllm_neuron_b200 import LLM, SamplingParams
    from vllm_neuron_b200.accuracy.kv_cache_analysis import (KVSnapshot, aggregate_kv_bc_across_prompts,
                                                             combined_bc_per_layer, compare_kv_caches,
                                                             extract_hf_kv, kv_report)

    path, hf = llama
    hf64 = copy.deepcopy(hf).double()
    llm = LLM(model=path, dtype="float32", max_model_len=256, max_num_seqs=2, max_num_batched_tokens=16,
              block_size=16, device="cpu")
    try:
        prompts = [[5, 9, 100, 7, 3], list(range(20, 45))]
        with KVSnapshot(llm.engine) as snap:
            outs = llm.generate(prompt_token_ids=prompts,
                                sampling_params=SamplingParams(temperature=0, max_tokens=4, ignore_eos=True))
        assert len(snap.kv) == 2
        raws = []
        for p, o in zip(prompts, outs):
            seq = p + list(o.outputs[0].token_ids)[:-1]
            ours = snap.kv[o.request_id]
            want = extract_hf_kv(hf, seq)
            assert set(ours) == set(want) and ours["layers.0.self_attn"][0].shape == want["layers.0.self_attn"][0].shape
            res = compare_kv_caches(want, ours)
            assert len(res) == len(seq)
            worst = max(m.k_linf for tok in res for hm in tok.values() for m in hm)
            assert worst < 1e-4, kv_report(res)
            res3, raw = compare_kv_caches(want, ours, baseline=extract_hf_kv(hf64, seq), return_raw_errors=True)
            assert "layers.0.self_attn._bc" in res3[0]
            raws.append(raw)
        agg = aggregate_kv_bc_across_prompts(raws, [len(p) for p in prompts])
        assert sorted(agg) == [0, 1, 2] and all(0.0 <= m.k_bc <= 1.0 for r in agg.values() for m in r.values())
        comb = combined_bc_per_layer(raws)
        assert sorted(comb) == sorted(snap.kv[outs[0].request_id])
        assert "layers.1.self_attn" in kv_report(res)
    finally:
        llm.shutdown()


def test_tensor_io_layout_and_hf_capture_alignment(llama, tmp_path):
    """Engine captures converted to the dp<N>/<pass>/<module>/rank<r>.pt layout, written and
    read back, then matched pass by pass (prefill, and decode by position) with an HF capture of
    the same prompt: every module output agrees."""
    from vllm_neuron_b200 import LLM, SamplingParams
    from vllm_neuron_b200.accuracy import tensor_io
    from vllm_neuron_b200.accuracy.tensor_alignment_utils import (align_and_truncate_hidden, count_real_tokens,
                                                                  match_passes, slice_token)

    path, hf = llama
    cap = str(tmp_path / "steps")
    nc = {"tensor_capture": {"modules": ["layers.0-1.mlp"], "capture_dir": cap}}
    llm = LLM(model=path, dtype="float32", max_model_len=128, max_num_seqs=1, block_size=16, device="cpu",
              additional_config={"neuron_config": nc})
    prompt = [4, 5, 6, 7, 8]
    llm.generate(prompt_token_ids=[prompt], sampling_params=SamplingParams(temperature=0, max_tokens=3,
                                                                           ignore_eos=True))
    llm.shutdown()
    ours = tensor_io.from_capture_steps(cap)
    assert [p.dir_name for p in ours] == ["prefill_s5_0", "decode_b1_1", "decode_b1_2"]
    assert ours[1].metadata.positions == [5]
    tensor_io.write(str(tmp_path / "io" / "dp0"), ours)
    back = tensor_io.read(str(tmp_path / "io"))
    assert [p.dir_name for p in back] == [p.dir_name for p in ours]
    assert torch.equal(back[0].tensors["layers.0.mlp"][0], ours[0].tensors["layers.0.mlp"][0])
    ref = tensor_io.capture_hf(hf, prompt, {"model.layers.0.mlp": "layers.0.mlp", "model.layers.1.mlp": "layers.1.mlp"},
                               max_new_tokens=4)
    pairs = match_passes(ref, back)
    assert len(pairs) == 3  # HF decoded one extra step: dropped
    for r, t in pairs:
        for name in ("layers.0.mlp", "layers.1.mlp"):
            (a, b), same = align_and_truncate_hidden(r.tensors[name][0], t.tensors[name][0])
            assert same and torch.allclose(a, b, atol=1e-4), (r.dir_name, name, (a - b).abs().max())
    assert count_real_tokens([0, 1, 2, 2, 2]) == 3 and slice_token(torch.zeros(1, 5, 8), 2).shape == (1, 1, 8)


def test_deterministic_replay_bitwise(llama, tmp_path):
    """Two fresh engines given the same seeded sampled workload produce the same tokens and
    bitwise-identical logit dumps (a replay check for races in the step pipeline)."""
    from vllm_neuron_b200 import LLM, SamplingParams
    from vllm_neuron_b200.engine.debug_logits import read_debug_logits

    path, _ = llama
    runs = []
    for i in range(2):
        d = str(tmp_path / f"run{i}")
        llm = LLM(model=path, dtype="float32", max_model_len=256, max_num_seqs=4, max_num_batched_tokens=32,
                  block_size=16, device="cpu", seed=3, additional_config={"neuron_config": {"debug_logits_dir": d}})
        try:
            outs = llm.generate(prompt_token_ids=[[5, 9, 100, 7, 3], list(range(20, 60)), [11] * 12],
                                sampling_params=SamplingParams(temperature=0.9, top_p=0.9, top_k=40, max_tokens=6,
                                                               ignore_eos=True, seed=17))
        finally:
            llm.shutdown()
        runs.append(([o.outputs[0].token_ids for o in outs], read_debug_logits(d)))
    (t0, l0), (t1, l1) = runs
    assert t0 == t1
    assert sorted(l0) == sorted(l1)
    for b in l0:
        assert sorted(l0[b]) == sorted(l1[b])
        assert all(torch.equal(l0[b][p], l1[b][p]) for p in l0[b])


def test_greedy_logit_gaps_zero_for_identical_engines(tmp_path):
    """The end-to-end greedy checker: an engine checked against itself has no gaps."""
    from vllm_neuron_b200 import LLM, SamplingParams
    from vllm_neuron_b200.accuracy.testing import greedy_logit_gaps, write_tiny_gpt_oss_checkpoint

    path = str(tmp_path / "ck")
    write_tiny_gpt_oss_checkpoint(path)
    llm = LLM(model=path, dtype="float32", device="cpu", max_model_len=256, max_num_seqs=2, block_size=16,
              additional_config={"neuron_config": {"quantization": "mxfp4"}})
    try:
        prompts = [[5, 6, 7, 8], list(range(100, 140))]
        outs = llm.generate(prompt_token_ids=prompts,
                            sampling_params=SamplingParams(temperature=0.0, max_tokens=4, ignore_eos=True))
        res = greedy_logit_gaps(llm.engine, prompts, [list(o.outputs[0].token_ids) for o in outs])
    finally:
        llm.shutdown()
    assert res.n_tokens == 8 and res.max_gap < 1e-4 and res.exact_fraction == 1.0
