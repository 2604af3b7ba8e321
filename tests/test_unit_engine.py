"""Block manager (prefix caching), scheduler policy and request lifecycle."""

import pytest
import torch

from vllm_neuron_b200.engine.block_manager import KVCacheManager
from vllm_neuron_b200.engine.request import Request, RequestStatus
from vllm_neuron_b200.engine.sampling_params import SamplingParams
from vllm_neuron_b200.engine.scheduler import Scheduler


def _req(i, n, max_tokens=4):
    return Request(f"r{i}", list(range(100 * i, 100 * i + n)), SamplingParams(temperature=0, max_tokens=max_tokens))


def test_block_allocation_and_free():
    kv = KVCacheManager(16, 4)
    r = _req(0, 10)
    assert kv.allocate_slots(r, 10)
    assert len(r.block_ids) == 3 and 0 not in r.block_ids
    free_before = kv.pool.num_free
    kv.free(r)
    assert kv.pool.num_free == free_before + 3


def test_prefix_cache_hit_and_eviction():
    kv = KVCacheManager(16, 4, enable_caching=True)
    a = Request("a", list(range(13)), SamplingParams())
    assert kv.allocate_slots(a, 13)
    a.num_computed_tokens = 13
    kv.cache_full_blocks(a)
    blocks_a = list(a.block_ids)
    kv.free(a)
    b = Request("b", list(range(12)) + [99, 98], SamplingParams())
    hit, n = kv.get_computed_blocks(b)
    assert n == 12 and hit == blocks_a[:3]
    b.num_computed_tokens = n
    assert kv.allocate_slots(b, 2, hit)
    assert b.block_ids[:3] == blocks_a[:3]
    # a prompt fully covered by cached blocks recomputes its last block
    c = Request("c", list(range(12)), SamplingParams())
    hit, n = kv.get_computed_blocks(c)
    assert n == 8


def test_scheduler_prefill_decode_separation_and_finish():
    kv = KVCacheManager(64, 4)
    s = Scheduler(kv, max_num_seqs=4, max_num_batched_tokens=16, max_model_len=64, max_num_prefills_per_step=1)
    r0, r1 = _req(0, 10, 2), _req(1, 20, 2)
    s.add_request(r0)
    s.add_request(r1)
    o = s.schedule()
    assert o.kind == "prefill" and [x.req_id for x in o.seqs] == ["r0"]
    s.update_from_output(o, {"r0": [7]})
    o = s.schedule()  # r1 prefill (segment 1 of 2): decode held back
    assert o.kind == "prefill" and o.seqs[0].req_id == "r1" and len(o.seqs[0].token_ids) == 16
    assert not o.seqs[0].sample
    s.update_from_output(o, {})
    o = s.schedule()
    assert o.kind == "prefill" and len(o.seqs[0].token_ids) == 4 and o.seqs[0].sample
    s.update_from_output(o, {"r1": [5]})
    o = s.schedule()
    assert o.kind == "decode" and {x.req_id for x in o.seqs} == {"r0", "r1"}
    done = s.update_from_output(o, {"r0": [8], "r1": [6]})
    assert {d.request_id for d in done} == {"r0", "r1"}
    assert all(d.status == RequestStatus.FINISHED_LENGTH for d in done)
    assert not s.has_unfinished()
    assert kv.pool.num_free == 63


def test_kv_admission_control():
    kv = KVCacheManager(9, 4)  # 8 usable blocks; max_model_len 16 -> 4 blocks each -> 2 concurrent
    s = Scheduler(kv, max_num_seqs=8, max_num_batched_tokens=64, max_model_len=16, max_num_prefills_per_step=4)
    for i in range(3):
        s.add_request(_req(i, 4, 8))
    o = s.schedule()
    assert len(o.seqs) == 2  # third request deferred by admission control


def test_stop_conditions():
    r = Request("x", [1, 2], SamplingParams(max_tokens=10, stop_token_ids=[42]), eos_token_id=7)
    r.output_token_ids = [3]
    assert not r.check_stop(100)
    r.output_token_ids.append(7)
    assert r.check_stop(100) and r.status == RequestStatus.FINISHED_STOPPED
    r2 = Request("y", [1], SamplingParams(max_tokens=10, ignore_eos=True), eos_token_id=7)
    r2.output_token_ids = [7]
    assert not r2.check_stop(100)
    r2.output_token_ids.append(42)
    assert not r2.check_stop(100)


@pytest.mark.parametrize("temperature", [0.0, 0.8])
def test_async_scheduling_matches_sync(temperature):
    """Asynchronous scheduling (step k+1 staged while step k runs, input tokens taken from
    the device) produces exactly the tokens of synchronous scheduling, including requests that
    stop early on a stop token and requests that arrive while others decode."""
    from vllm_neuron_b200 import LLM, SamplingParams
    from tiny_configs import TINY_GPT_OSS, workload

    prompts = workload(n=5, lo=8, hi=40)
    outs = {}
    for mode in (False, True):
        llm = LLM(hf_config=dict(TINY_GPT_OSS), load_format="dummy", dtype="float32", max_model_len=256,
                  max_num_seqs=8, max_num_batched_tokens=128, block_size=16, device="cpu", seed=11,
                  async_scheduling=mode, additional_config={"neuron_config": {"quantization": "bf16"}})
        sps = [SamplingParams(temperature=temperature, max_tokens=12 + i, ignore_eos=True, seed=3,
                              stop_token_ids=[7] if i == 2 else None) for i in range(len(prompts))]
        eng = llm.engine
        for i, p in enumerate(prompts[:3]):
            eng.add_request(f"a{i}", p, sps[i])
        res = {}
        steps = 0
        while eng.has_unfinished_requests():
            for o in eng.step():
                if o.finished:
                    res[o.request_id] = o.outputs[0].token_ids
            steps += 1
            if steps == 6:  # late arrivals join while the first requests decode
                for i, p in enumerate(prompts[3:], start=3):
                    eng.add_request(f"a{i}", p, sps[i])
        outs[mode] = res
        assert eng._inflight is None
        if mode:
            assert eng.async_stats["lookahead"] > 10, eng.async_stats
            assert eng.async_stats["sync_fallback"] > 0  # prefills run synchronously
            from prometheus_client import REGISTRY

            got = REGISTRY.get_sample_value("vllm_b200:async_steps_total", {"model_name": "model", "mode": "lookahead"})
            assert got is not None and got >= eng.async_stats["lookahead"]
        llm.shutdown()
    assert outs[True] == outs[False]


@pytest.mark.parametrize("tp", [1, 2])
def test_logprobs_match_reference(tmp_path, tp):
    """Top-N logprobs of the raw logits and the sampled token's logprob, over the vocab shards
    (TP=2 gathers them), against HF transformers' log-softmax at every generated position."""
    from transformers import LlamaConfig, LlamaForCausalLM

    from vllm_neuron_b200 import LLM, SamplingParams
    from vllm_neuron_b200.utils.checkpoints import save_state_dict

    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=1001, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=256,
                      tie_word_embeddings=False)
    cfg._attn_implementation = "eager"
    hf = LlamaForCausalLM(cfg).eval().float()
    d = cfg.to_dict()
    d["architectures"] = ["LlamaForCausalLM"]
    save_state_dict({k: v.detach().clone().contiguous() for k, v in hf.state_dict().items()}, str(tmp_path), d)
    prompt = [5, 17, 300, 42, 7, 999]
    llm = LLM(model=str(tmp_path), dtype="float32", max_model_len=128, max_num_seqs=2, max_num_batched_tokens=64,
              block_size=16, device="cpu", tensor_parallel_size=tp)
    try:
        out = llm.generate(prompt_token_ids=[prompt],
                           sampling_params=SamplingParams(temperature=0.7, seed=3, max_tokens=5, ignore_eos=True,
                                                          logprobs=3))[0].outputs[0]
    finally:
        llm.shutdown()
    assert len(out.logprobs) == len(out.token_ids) == 5
    ids = torch.tensor([prompt + out.token_ids[:-1]])
    with torch.no_grad():
        lp = torch.log_softmax(hf(ids).logits[0, len(prompt) - 1:].float(), -1)
    for j, (t, entry) in enumerate(zip(out.token_ids, out.logprobs)):
        assert abs(entry[t] - lp[j, t].item()) < 1e-3
        top = lp[j].topk(3)
        for v, i in zip(top.values.tolist(), top.indices.tolist()):
            assert abs(entry[i] - v) < 1e-3, (j, i, entry)


def test_parallel_sampling_n(tmp_path):
    """n > 1: n completions per prompt with distinct samples; greedy children agree."""
    from vllm_neuron_b200 import LLM, SamplingParams

    llm = LLM(hf_config={"architectures": ["LlamaForCausalLM"], "vocab_size": 512, "hidden_size": 64,
                         "intermediate_size": 128, "num_hidden_layers": 2, "num_attention_heads": 4,
                         "num_key_value_heads": 2, "max_position_embeddings": 256},
              load_format="dummy", dtype="float32", max_model_len=256, max_num_seqs=8, max_num_batched_tokens=256,
              block_size=16, device="cpu", enable_prefix_caching=True)
    try:
        outs = llm.generate(prompt_token_ids=[[1, 2, 3, 4], [9, 8]],
                            sampling_params=[SamplingParams(n=4, temperature=1.0, seed=1, max_tokens=8,
                                                            ignore_eos=True),
                                             SamplingParams(n=2, temperature=0, max_tokens=8, ignore_eos=True)])
    finally:
        llm.shutdown()
    assert [len(o.outputs) for o in outs] == [4, 2]
    assert [c.index for c in outs[0].outputs] == [0, 1, 2, 3]
    assert len({tuple(c.token_ids) for c in outs[0].outputs}) > 1
    assert outs[1].outputs[0].token_ids == outs[1].outputs[1].token_ids


def test_sliding_window_kv_group_frees_blocks_behind_the_window():
    """Hybrid KV groups: the windowed layers' table returns every block wholly behind the
    window of the step's first query (keys j > p - W stay visible) to its own pool, so a long
    sequence holds about W / block_size + 1 windowed blocks while the full-attention table
    keeps the whole context."""
    from vllm_neuron_b200.engine.block_manager import KVCacheManager
    from vllm_neuron_b200.engine.request import Request
    from vllm_neuron_b200.engine.sampling_params import SamplingParams

    bs, W = 16, 128
    kv = KVCacheManager(200, bs, False, sliding_window=W, swa_blocks=40)
    req = Request("r", list(range(300)), SamplingParams(max_tokens=500))
    assert kv.allocate_slots(req, 300)  # prefill: every block of the prompt in both groups
    assert len(req.block_ids) == len(req.swa_block_ids) == 19 and kv.swa_pool.num_free == 40 - 1 - 19
    req.num_computed_tokens = 300
    for _ in range(200):  # decode: one token per step
        assert kv.allocate_slots(req, 1)
        p = req.num_computed_tokens
        live = [b for b in req.swa_block_ids if b != 0]
        first_visible = p - W + 1  # the query at p sees keys > p - W
        # every block holding a visible key is live, every freed one is wholly behind the window
        assert all(req.swa_block_ids[j] != 0 for j in range(first_visible // bs, -(-(p + 1) // bs)))
        assert all((j + 1) * bs <= first_visible for j, b in enumerate(req.swa_block_ids) if b == 0)
        assert len(live) <= W // bs + 2
        req.num_computed_tokens += 1
    assert len(req.block_ids) == -(-500 // bs)  # the full group keeps everything
    kv.free(req)
    assert kv.swa_pool.num_free == 39 and kv.pool.num_free == 199 and req.swa_block_ids == []


def test_mixed_prefill_decode_steps_keep_greedy_tokens(monkeypatch):
    """With mixed_prefill_tokens, prompt chunks ride along in the decode steps of running
    requests ("mixed" steps: decodes first, then chunks of at most that many prompt tokens);
    greedy tokens equal the separate-steps engine's."""
    from tiny_configs import workload

    from vllm_neuron_b200 import LLM, SamplingParams
    from vllm_neuron_b200.accuracy.testing import TINY_GPT_OSS_D64
    from vllm_neuron_b200.engine import model_runner

    kinds, launched = [], []
    orig, orig_launch = model_runner.ModelRunner.execute, model_runner.ModelRunner.launch

    def spy(self, so, *a, **k):
        kinds.append((so.kind, so.num_decode, sum(len(s.token_ids) for s in so.seqs[so.num_decode:])))
        return orig(self, so, *a, **k)

    def spy_launch(self, so, *a, **k):
        launched.append(so.kind)
        return orig_launch(self, so, *a, **k)

    monkeypatch.setattr(model_runner.ModelRunner, "execute", spy)
    monkeypatch.setattr(model_runner.ModelRunner, "launch", spy_launch)
    cfg = dict(TINY_GPT_OSS_D64)
    cfg["architectures"] = ["GptOssForCausalLM"]
    outs = []
    for mixed, async_ in ((0, False), (32, False), (32, True)):
        llm = LLM(hf_config=dict(cfg), load_format="dummy", dtype="float32", device="cpu", max_model_len=512,
                  max_num_seqs=4, max_num_batched_tokens=128, block_size=16, seed=2, mixed_prefill_tokens=mixed,
                  async_scheduling=async_)
        try:
            o = llm.generate(prompt_token_ids=workload(n=7, lo=20, hi=150, vocab=4000, seed=3),
                             sampling_params=SamplingParams(temperature=0, max_tokens=10, ignore_eos=True))
            outs.append([x.outputs[0].token_ids for x in o])
        finally:
            llm.shutdown()
    mixed_steps = [k for k in kinds if k[0] == "mixed"]
    assert mixed_steps and all(d > 0 and 0 < n <= 32 for _, d, n in mixed_steps), kinds
    assert outs[0] == outs[1] == outs[2]
    assert "mixed" in launched, launched  # asynchronous mixed steps
