"""Disaggregated prefill/decode (1P1D) on CPU with the synthetic KV-verifying model: the
decode engine must find every prompt position's KV exactly as the prefill engine wrote it,
across different TP degrees on the two sides; a transfer that never arrives aborts the
request within the connector timeout instead of blocking the engine."""

import os

import time

import pytest

SYN = {"architectures": ["SyntheticModel"], "num_hidden_layers": 3, "num_key_value_heads": 4, "head_dim": 16,
       "vocab_size": 32, "max_position_embeddings": 1024}


@pytest.fixture(autouse=True)
def _synthetic(monkeypatch):
    monkeypatch.setenv("VLLM_B200_SYNTHETIC_MODEL", "1")
    monkeypatch.setenv("VLLM_NEURON_SYNTHETIC_MODEL", "1")


def _llm(role, store, tp=1, timeout=30.0, block_size=16):
    from vllm_neuron_b200 import LLM

    return LLM(hf_config=dict(SYN), load_format="dummy", dtype="bfloat16", max_model_len=256, max_num_seqs=4,
               max_num_batched_tokens=256, block_size=block_size, device="cpu", tensor_parallel_size=tp,
               kv_transfer_config={"kv_connector": "HostStagedConnector", "kv_role": role,
                                   "kv_connector_extra_config": {"store_path": store, "timeout_s": timeout}})


@pytest.mark.parametrize("p_tp,d_tp,d_bs", [(1, 1, 16), (2, 1, 32), (1, 2, 16)])
def test_one_prefill_one_decode(tmp_path, p_tp, d_tp, d_bs):
    from vllm_neuron_b200 import SamplingParams
    from vllm_neuron_b200.models.synthetic import TOKEN_EMPTY, TOKEN_SUCCESS

    store = str(tmp_path / "kv")
    prompts = [list(range(1, 40)), list(range(3, 100)), [9, 8, 7]]
    prefill = _llm("kv_producer", store, p_tp)
    try:
        outs = prefill.generate([{"prompt_token_ids": p, "kv_transfer_params": {"do_remote_decode": True}}
                                 for p in prompts], SamplingParams(temperature=0, max_tokens=1, ignore_eos=True))
    finally:
        prefill.shutdown()
    params = [o.kv_transfer_params for o in outs]
    assert all(p and p["do_remote_prefill"] for p in params)
    assert [o.outputs[0].token_ids for o in outs] == [[TOKEN_EMPTY]] * 3  # P computed from position 0
    decode = _llm("kv_consumer", store, d_tp, block_size=d_bs)
    try:
        outs2 = decode.generate([{"prompt_token_ids": p, "kv_transfer_params": kp} for p, kp in zip(prompts, params)],
                                SamplingParams(temperature=0, max_tokens=4, ignore_eos=True))
        st = decode.engine.connector.stats
    finally:
        decode.shutdown()
    for o, p in zip(outs2, prompts):
        assert o.outputs[0].token_ids == [TOKEN_SUCCESS] * 4, o.outputs[0].token_ids
        assert o.num_cached_tokens == len(p) - 1  # only the last prompt token was computed on D
    assert st["loaded"] == 3


def test_missing_transfer_aborts_request(tmp_path):
    from vllm_neuron_b200 import SamplingParams

    store = str(tmp_path / "kv")
    os.makedirs(store)
    decode = _llm("kv_consumer", store, 1, timeout=0.5)
    try:
        bogus = {"do_remote_prefill": True, "transfer_id": "nope", "num_tokens": 20, "remote_tp_size": 1}
        outs = decode.generate([{"prompt_token_ids": list(range(20)), "kv_transfer_params": bogus},
                                {"prompt_token_ids": list(range(5, 15))}],
                               SamplingParams(temperature=0, max_tokens=2, ignore_eos=True))
    finally:
        decode.shutdown()
    assert outs[0].outputs[0].finish_reason == "abort" and outs[0].outputs[0].token_ids == []
    assert len(outs[1].outputs[0].token_ids) == 2  # the engine kept serving


def test_corrupted_transfer_is_detected(tmp_path):
    """A transfer whose KV was tampered with (a flipped value) is reported as KV_MISMATCH."""
    import torch

    from vllm_neuron_b200 import SamplingParams
    from vllm_neuron_b200.models.synthetic import TOKEN_FAIL

    store = str(tmp_path / "kv")
    prefill = _llm("kv_producer", store)
    try:
        o = prefill.generate([{"prompt_token_ids": list(range(1, 30)), "kv_transfer_params": {"do_remote_decode": True}}],
                             SamplingParams(temperature=0, max_tokens=1, ignore_eos=True))[0]
    finally:
        prefill.shutdown()
    kp = o.kv_transfer_params
    path = os.path.join(store, f"{kp['transfer_id']}.rank0.pt")
    blob = torch.load(path, weights_only=False)
    blob["layers"][1][0][7, 2, 3] += 1  # one value of layer 1, key, position 7
    torch.save(blob, path)
    decode = _llm("kv_consumer", store)
    try:
        o2 = decode.generate([{"prompt_token_ids": list(range(1, 30)), "kv_transfer_params": kp}],
                             SamplingParams(temperature=0, max_tokens=2, ignore_eos=True))[0]
    finally:
        decode.shutdown()
    assert o2.outputs[0].token_ids == [TOKEN_FAIL, TOKEN_FAIL]


def test_proxy_routes_prefill_then_decode(tmp_path):
    from fastapi.testclient import TestClient

    from vllm_neuron_b200.engine.async_engine import AsyncLLM
    from vllm_neuron_b200.entrypoints.disagg_proxy import build_proxy
    from vllm_neuron_b200.entrypoints.openai_server import build_app
    from vllm_neuron_b200.models.synthetic import TOKEN_SUCCESS

    store = str(tmp_path / "kv")

    def eng(role):
        return AsyncLLM(hf_config=dict(SYN), load_format="dummy", dtype="bfloat16", max_model_len=256,
                        max_num_seqs=4, max_num_batched_tokens=256, block_size=16, device="cpu",
                        kv_transfer_config={"kv_connector": "HostStagedConnector", "kv_role": role,
                                            "kv_connector_extra_config": {"store_path": store}})

    pe, de = eng("kv_producer"), eng("kv_consumer")
    try:
        with TestClient(build_app(pe, "syn")) as pc, TestClient(build_app(de, "syn")) as dc:
            routes = {"http://p": pc, "http://d": dc}

            async def post(url, body):
                base, path = url.split("/v1/")
                return routes[base].post("/v1/" + path, json=body).json()

            with TestClient(build_proxy("http://p", "http://d", post)) as proxy:
                r = proxy.post("/v1/completions", json={"prompt": list(range(1, 50)), "max_tokens": 3,
                                                         "temperature": 0, "ignore_eos": True}).json()
                assert r["choices"][0]["token_ids"] == [TOKEN_SUCCESS] * 3
                assert proxy.get("/health").json()["transfers"] == 1
    finally:
        pe.shutdown()
        de.shutdown()


def test_decode_bench_connector_skips_prefill(tmp_path):
    """Decode-only benchmarking: every prompt is admitted as prefilled (its KV filled with
    noise), so each request computes only its last prompt token and then decodes."""
    from vllm_neuron_b200 import LLM, SamplingParams

    llm = LLM(hf_config={"architectures": ["LlamaForCausalLM"], "vocab_size": 512, "hidden_size": 64,
                         "intermediate_size": 128, "num_hidden_layers": 2, "num_attention_heads": 4,
                         "num_key_value_heads": 2, "max_position_embeddings": 256},
              load_format="dummy", dtype="float32", max_model_len=256, max_num_seqs=4, max_num_batched_tokens=256,
              block_size=16, device="cpu",
              kv_transfer_config={"kv_connector": "NeuronDecodeBenchConnector", "kv_role": "kv_consumer"})
    prompts = [list(range(1, 100)), list(range(5, 40))]
    try:
        outs = llm.generate(prompt_token_ids=prompts,
                            sampling_params=SamplingParams(temperature=0, max_tokens=5, ignore_eos=True))
        st = llm.engine.connector.stats
    finally:
        llm.shutdown()
    for o, p in zip(outs, prompts):
        assert len(o.outputs[0].token_ids) == 5
        assert o.num_cached_tokens == len(p) - 1
    assert st["loaded"] == 2


def test_bidirectional_kv_multi_turn(tmp_path, monkeypatch):
    """Two conversation turns over 1P1D with decode -> prefill KV: after turn 1 the decode
    engine exports the conversation so far; turn 2's prefill engine (kv_both) loads that prefix
    (checked byte-exact by the synthetic model) and computes only the new tokens, then hands the
    whole prompt to the decode engine.  A transfer whose tokens do not match the prompt is
    ignored and the prompt computed locally."""
    from vllm_neuron_b200 import SamplingParams
    from vllm_neuron_b200.models.synthetic import TOKEN_EMPTY, TOKEN_SUCCESS

    monkeypatch.setenv("VLLM_B200_BIDIRECTIONAL_KV", "1")
    store = str(tmp_path / "kv")
    sp1 = SamplingParams(temperature=0, max_tokens=1, ignore_eos=True)
    sp4 = SamplingParams(temperature=0, max_tokens=4, ignore_eos=True)
    prefill, decode = _llm("kv_both", store), _llm("kv_consumer", store)
    try:
        turn1 = list(range(1, 30))
        p1 = prefill.generate([{"prompt_token_ids": turn1, "kv_transfer_params": {"do_remote_decode": True}}], sp1)
        assert p1[0].outputs[0].token_ids == [TOKEN_EMPTY]
        # without ``return_kv`` the decode engine exports nothing when the request finishes
        d0 = decode.generate([{"prompt_token_ids": turn1, "kv_transfer_params": p1[0].kv_transfer_params}], sp4)
        assert not d0[0].kv_transfer_params and decode.engine.connector.stats["exported"] == 0
        p1 = prefill.generate([{"prompt_token_ids": turn1, "kv_transfer_params": {"do_remote_decode": True}}], sp1)
        d1 = decode.generate([{"prompt_token_ids": turn1,
                               "kv_transfer_params": {**p1[0].kv_transfer_params, "return_kv": True}}], sp4)
        out1 = list(d1[0].outputs[0].token_ids)
        assert out1 == [TOKEN_SUCCESS] * 4
        back = d1[0].kv_transfer_params
        assert decode.engine.connector.exported[-1][1] - time.monotonic() <= 60.0  # the short return TTL
        assert back and back["do_remote_prefill"] and back["num_tokens"] == len(turn1) + 3
        # turn 2: the conversation so far plus the user's new tokens
        turn2 = turn1 + out1 + [11, 12, 13, 14, 15]
        p2 = prefill.generate([{"prompt_token_ids": turn2, "kv_transfer_params": {**back, "do_remote_decode": True}}],
                              sp1)
        assert p2[0].num_cached_tokens == len(turn1) + 3  # the prefix came from the decode engine
        assert p2[0].outputs[0].token_ids == [TOKEN_SUCCESS]  # and it verified byte-exact
        assert prefill.engine.connector.stats["loaded"] == 1
        d2 = decode.generate([{"prompt_token_ids": turn2, "kv_transfer_params": p2[0].kv_transfer_params}], sp4)
        assert d2[0].outputs[0].token_ids == [TOKEN_SUCCESS] * 4
        # a prompt that does not extend the transferred conversation ignores the transfer
        other = [7] * 40
        p3 = prefill.generate([{"prompt_token_ids": other, "kv_transfer_params": {**back, "do_remote_decode": True}}],
                              sp1)
        assert p3[0].num_cached_tokens == 0 and prefill.engine.connector.stats["loaded"] == 1
    finally:
        prefill.shutdown()
        decode.shutdown()


def test_streamed_response_carries_kv_transfer_params(tmp_path):
    """A prefill server's streamed completion ends with a chunk that carries the
    kv_transfer_params (non-streamed: in the response body)."""
    import json

    from fastapi.testclient import TestClient

    from vllm_neuron_b200.engine.async_engine import AsyncLLM
    from vllm_neuron_b200.entrypoints.openai_server import build_app

    store = str(tmp_path / "kv")
    eng = AsyncLLM(hf_config=dict(SYN), load_format="dummy", dtype="bfloat16", max_model_len=256, max_num_seqs=4,
                   max_num_batched_tokens=256, block_size=16, device="cpu",
                   kv_transfer_config={"kv_connector": "HostStagedConnector", "kv_role": "kv_producer",
                                       "kv_connector_extra_config": {"store_path": store}})
    try:
        with TestClient(build_app(eng, "syn")) as c:
            body = {"model": "syn", "prompt": list(range(1, 30)), "max_tokens": 1, "temperature": 0,
                    "kv_transfer_params": {"do_remote_decode": True}}
            plain = c.post("/v1/completions", json=body).json()
            assert plain["kv_transfer_params"]["do_remote_prefill"]
            chunks = []
            with c.stream("POST", "/v1/completions", json=dict(body, stream=True)) as resp:
                for line in resp.iter_lines():
                    if line.startswith("data: {"):
                        chunks.append(json.loads(line[6:]))
            assert chunks and chunks[-1]["kv_transfer_params"]["do_remote_prefill"]
            assert all("kv_transfer_params" not in ch for ch in chunks[:-1])
    finally:
        eng.shutdown()
