"""OpenAI-compatible server on the tiny GPT-OSS model (CPU): completions (plain and
streamed, token-id prompts), models, health, metrics; plus the CLI argument mapping."""

import json

import pytest

from tiny_configs import TINY_GPT_OSS


@pytest.fixture(scope="module")
def client():
    from fastapi.testclient import TestClient

    from vllm_neuron_b200.engine.async_engine import AsyncLLM
    from vllm_neuron_b200.entrypoints.openai_server import build_app

    eng = AsyncLLM(hf_config=dict(TINY_GPT_OSS), load_format="dummy", dtype="float32", max_model_len=256,
                   max_num_seqs=4, max_num_batched_tokens=128, block_size=16, device="cpu",
                   additional_config={"neuron_config": {"quantization": "bf16"}})
    with TestClient(build_app(eng, "tiny")) as c:
        c.b200_engine = eng
        yield c
    eng.shutdown()


def test_health_models_metrics(client):
    assert client.get("/health").json()["status"] == "ok"
    assert client.get("/v1/models").json()["data"][0]["id"] == "tiny"
    assert client.get("/metrics").status_code == 200


def test_completion_and_stream_agree(client):
    body = {"prompt": [5, 6, 7, 8, 9], "max_tokens": 6, "temperature": 0, "ignore_eos": True}
    r = client.post("/v1/completions", json=body).json()
    toks = r["choices"][0]["token_ids"]
    assert len(toks) == 6 and r["usage"]["completion_tokens"] == 6
    streamed = []
    with client.stream("POST", "/v1/completions", json=dict(body, stream=True)) as resp:
        for line in resp.iter_lines():
            if line.startswith("data:") and not line.endswith("[DONE]"):
                streamed += json.loads(line[5:])["choices"][0]["token_ids"]
    assert streamed == toks


def test_cli_engine_kwargs():
    import argparse

    from vllm_neuron_b200.entrypoints import cli

    ap = argparse.ArgumentParser()
    cli._engine_args(ap)
    a = ap.parse_args(["/m", "-tp", "8", "--max-num-seqs", "64",
                       "--additional-config", '{"neuron_config": {"ep_degree": 8}}'])
    kw = cli.engine_kwargs(a)
    assert kw["tensor_parallel_size"] == 8 and kw["additional_config"]["neuron_config"]["ep_degree"] == 8


def test_profile_endpoints(client, tmp_path, monkeypatch):
    monkeypatch.setattr(client.b200_engine.engine.profiler.cfg, "output_dir", str(tmp_path))
    r = client.post("/start_profile")
    assert r.json()["status"] == "started"
    assert client.post("/start_profile").status_code == 400  # already running
    client.post("/v1/completions", json={"prompt": [5, 6, 7], "max_tokens": 2, "temperature": 0})
    r = client.post("/stop_profile").json()
    assert r["status"] == "stopped" and r["steps"] >= 2
    import os

    assert os.path.exists(r["trace"]) and os.path.exists(r["summary"])
    assert os.path.dirname(r["trace"]) == str(tmp_path)
    assert client.post("/stop_profile").status_code == 400


def test_profiler_config_aliases():
    from vllm_neuron_b200.profiler import ProfilerConfig

    c = ProfilerConfig.from_dict({"activities": ["device_profile", "system_profile"], "output_dir": "/tmp/x",
                                  "neuron_cores": [0]})
    assert c.activities == ["cpu", "cuda"] and c.output_dir == "/tmp/x"
    with pytest.raises(ValueError):
        ProfilerConfig.from_dict({"activities": ["npu"]})


def test_structured_output_request_fields():
    from vllm_neuron_b200.entrypoints.openai_server import _sampling_from

    def so(body):
        p = _sampling_from(body).structured_outputs
        return None if p is None else (p.json, p.regex, p.choice, p.grammar, p.json_object)

    assert so({}) is None
    assert so({"response_format": {"type": "json_object"}}) == (None, None, None, None, True)
    schema = {"type": "object"}
    assert so({"response_format": {"type": "json_schema", "json_schema": {"name": "x", "schema": schema}}})[0] == schema
    assert so({"guided_regex": "a+"})[1] == "a+"
    assert so({"guided_choice": ["a", "b"]})[2] == ["a", "b"]
    assert so({"structured_outputs": {"grammar": 'root ::= "x"'}})[3] == 'root ::= "x"'


def test_logprobs_request_and_payload():
    from vllm_neuron_b200.entrypoints.openai_server import _logprobs_from, _logprobs_payload

    assert _logprobs_from({}) is None and _logprobs_from({"logprobs": 2}) == 2
    assert _logprobs_from({"logprobs": True, "top_logprobs": 3}) == 3
    detok = lambda ids: "".join(chr(97 + i) for i in ids)  # noqa: E731
    entries = [{1: -0.1, 2: -2.0}, {0: -0.5}]
    comp = _logprobs_payload([1, 0], entries, detok, chat=False)
    assert comp["tokens"] == ["b", "a"] and comp["token_logprobs"] == [-0.1, -0.5]
    chat = _logprobs_payload([1, 0], entries, detok, chat=True)
    assert chat["content"][0]["top_logprobs"] == [{"token": "c", "logprob": -2.0}]
