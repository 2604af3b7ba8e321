"""Structured outputs on CPU: a tiny random Llama with a word-level tokenizer saved next to it;
every constrained request's text must satisfy its regex / choice / grammar, at TP=1 and TP=2
(gloo), greedy and sampled; constrained requests are refused when the feature is off."""

import json
import re

import pytest
import torch

V = 512
TOKS = [str(d) for d in range(10)] + list('{}":, ') + [chr(ord("a") + i) for i in range(26)] + ["true", "false", "null"]
TOKS += ["[", "]"]
TOKS += [f"<x{i}>" for i in range(V - len(TOKS) - 2)] + ["<unk>", "</s>"]
EOS = V - 1


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    from tokenizers import Tokenizer, decoders, models
    from transformers import LlamaConfig, LlamaForCausalLM, PreTrainedTokenizerFast

    from vllm_neuron_b200.utils.checkpoints import save_state_dict

    path = tmp_path_factory.mktemp("so")
    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=V, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=256,
                      tie_word_embeddings=False, eos_token_id=EOS)
    m = LlamaForCausalLM(cfg).eval().float()
    d = cfg.to_dict()
    d["architectures"] = ["LlamaForCausalLM"]
    save_state_dict({k: v.detach().clone().contiguous() for k, v in m.state_dict().items()}, str(path), d)
    tk = Tokenizer(models.WordLevel({t: i for i, t in enumerate(TOKS)}, unk_token="<unk>"))
    tk.decoder = decoders.Fuse()  # detokenised text joins the tokens as they are
    PreTrainedTokenizerFast(tokenizer_object=tk, eos_token="</s>", unk_token="<unk>").save_pretrained(str(path))
    return str(path)


def _text(ids):
    return "".join(TOKS[i] for i in ids if i != EOS)


def _llm(path, tp=1, enabled=True):
    from vllm_neuron_b200 import LLM

    return LLM(model=path, dtype="float32", max_model_len=128, max_num_seqs=4, max_num_batched_tokens=64,
               block_size=16, device="cpu", tensor_parallel_size=tp,
               additional_config={"neuron_config": {"enable_structured_outputs": enabled}})


CASES = [({"regex": "[a-c]{3}[0-9]{2}"}, lambda s: re.fullmatch("[a-c]{3}[0-9]{2}", s)),
         ({"choice": ["yes", "no", "maybe"]}, lambda s: s in ("yes", "no", "maybe")),
         ({"grammar": 'root ::= "{" [a-z] ":" [0-9] "}"'}, lambda s: re.fullmatch(r"\{[a-z]:[0-9]\}", s))]


@pytest.mark.parametrize("tp", [1, 2])
def test_constrained_outputs_follow_their_grammar(ckpt, tp):
    from vllm_neuron_b200 import SamplingParams

    llm = _llm(ckpt, tp)
    prompts = [[11, 12, 13, 14, 20 + i] for i in range(len(CASES) * 2)]
    params = []
    for i in range(len(prompts)):
        so, _ = CASES[i % len(CASES)]
        params.append(SamplingParams(temperature=0 if i < len(CASES) else 0.9, seed=i, max_tokens=32,
                                     structured_outputs=so))
    try:
        outs = llm.generate(prompt_token_ids=prompts, sampling_params=params)
        free = llm.generate(prompt_token_ids=[prompts[0]],
                            sampling_params=SamplingParams(temperature=0, max_tokens=8, ignore_eos=True))
    finally:
        llm.shutdown()
    for i, o in enumerate(outs):
        text = _text(o.outputs[0].token_ids)
        assert CASES[i % len(CASES)][1](text), (i, text, o.outputs[0].token_ids)
        assert o.outputs[0].finish_reason == "stop", o.outputs[0].finish_reason
    assert len(free[0].outputs[0].token_ids) == 8  # an unconstrained request in the same engine


def test_refused_when_disabled(ckpt):
    from vllm_neuron_b200 import SamplingParams

    llm = _llm(ckpt, enabled=False)
    try:
        with pytest.raises(ValueError, match="structured outputs are disabled"):
            llm.generate(prompt_token_ids=[[1, 2, 3]],
                         sampling_params=SamplingParams(max_tokens=4, structured_outputs={"regex": "a+"}))
    finally:
        llm.shutdown()


def test_json_schema_bitmask():
    import xgrammar as xgr

    from vllm_neuron_b200.engine.structured_output import (StructuredOutputManager, StructuredOutputsParams,
                                                            mask_logits)

    mgr = StructuredOutputManager(xgr.TokenizerInfo(TOKS, stop_token_ids=[EOS]))
    schema = {"type": "object", "properties": {"a": {"type": "integer"}}, "required": ["a"]}
    m = mgr.matcher(StructuredOutputsParams.from_any({"json": json.dumps(schema)}))
    for t in '{"a":12}':  # drive the matcher through a valid document, token by token
        bm = mgr.bitmask([m])
        logits = mask_logits(torch.zeros(1, V), bm, 0)
        assert torch.isfinite(logits[0, TOKS.index(t)]), t
        assert m.accept_token(TOKS.index(t))
    bm = mgr.bitmask([m, None])
    allowed = torch.isfinite(mask_logits(torch.zeros(2, V), bm, 0))
    assert allowed[0, EOS] and not allowed[0, TOKS.index("a")]
    assert allowed[1].all()  # rows without a grammar are unconstrained
    # a vocabulary shard (TP): ids [256, 512) see the same bits
    assert torch.equal(torch.isfinite(mask_logits(torch.zeros(2, 256), bm, 256)), allowed[:, 256:])


@pytest.mark.parametrize("include", [False, True])
def test_stop_strings_cut_generation(ckpt, include):
    from transformers import AutoTokenizer

    from vllm_neuron_b200 import SamplingParams

    tok = AutoTokenizer.from_pretrained(ckpt)
    llm = _llm(ckpt, enabled=False)
    prompt = [11, 12, 13, 14, 30]
    try:
        full = llm.generate(prompt_token_ids=[prompt],
                            sampling_params=SamplingParams(temperature=0, max_tokens=20, ignore_eos=True))[0]
        ids = full.outputs[0].token_ids
        text = tok.decode(ids, skip_special_tokens=True)
        stop = tok.decode(ids[4:6], skip_special_tokens=True)
        cut = llm.generate(prompt_token_ids=[prompt],
                           sampling_params=SamplingParams(temperature=0, max_tokens=20, ignore_eos=True, stop=[stop],
                                                          include_stop_str_in_output=include))[0].outputs[0]
    finally:
        llm.shutdown()
    p = text.find(stop)
    assert cut.finish_reason == "stop" and len(cut.token_ids) <= 6
    assert cut.text == text[:p + (len(stop) if include else 0)]


def test_tool_calls_required_and_named_through_the_server(ckpt):
    """tool_choice="required" constrains the output to a list of {name, parameters} over the
    declared tools; a named tool constrains it to that tool's arguments.  Both come back as
    message.tool_calls with finish_reason "tool_calls"."""
    from fastapi.testclient import TestClient

    from vllm_neuron_b200.engine.async_engine import AsyncLLM
    from vllm_neuron_b200.entrypoints.openai_server import build_app

    tools = [{"type": "function", "function": {"name": "ab", "parameters": {
        "type": "object", "properties": {"x": {"type": "integer"}}, "required": ["x"]}}},
             {"type": "function", "function": {"name": "cd", "parameters": {
                 "type": "object", "properties": {"y": {"type": "boolean"}}, "required": ["y"]}}}]
    eng = AsyncLLM(model=ckpt, dtype="float32", max_model_len=128, max_num_seqs=4, max_num_batched_tokens=64,
                   block_size=16, device="cpu", additional_config={"neuron_config": {"enable_structured_outputs": True}})
    try:
        with TestClient(build_app(eng, "so")) as c:
            msgs = [{"role": "user", "content": "a b c"}]
            r = c.post("/v1/chat/completions", json={"model": "so", "messages": msgs, "tools": tools,
                                                     "tool_choice": "required", "max_tokens": 60,
                                                     "temperature": 0}).json()
            ch = r["choices"][0]
            if ch["finish_reason"] == "tool_calls":
                calls = ch["message"]["tool_calls"]
                assert calls and all(t["function"]["name"] in ("ab", "cd") for t in calls)
                for t in calls:
                    args = json.loads(t["function"]["arguments"])
                    assert ("x" in args) if t["function"]["name"] == "ab" else ("y" in args)
            else:
                # a random model may keep appending calls until max_tokens (the array is
                # unbounded, as in vLLM); every item it wrote still follows the tool schemas
                assert ch["finish_reason"] == "length", ch
                item = r'\{"name": "(ab|cd)", "parameters": \{("x": -?\d+|"y": (true|false))\}\}'
                assert re.match(r"\[" + item + r"(, " + item + r")*", ch["message"]["content"]), ch
            r = c.post("/v1/chat/completions", json={"model": "so", "messages": msgs, "tools": tools,
                                                     "tool_choice": {"type": "function", "function": {"name": "cd"}},
                                                     "max_tokens": 40, "temperature": 0}).json()
            call = r["choices"][0]["message"]["tool_calls"][0]
            assert call["function"]["name"] == "cd" and isinstance(json.loads(call["function"]["arguments"])["y"], bool)
            bad = c.post("/v1/chat/completions", json={"model": "so", "messages": msgs, "tools": tools,
                                                       "tool_choice": {"type": "function", "function": {"name": "zz"}}})
            assert bad.status_code == 400
    finally:
        eng.shutdown()


def test_tool_call_parsers():
    """auto tool choice: calls read back from GPT-OSS harmony text, Hermes blocks and bare JSON."""
    from vllm_neuron_b200.entrypoints.tool_calls import parse_tool_calls

    tools = [{"type": "function", "function": {"name": "get_weather", "parameters": {}}}]
    harmony = ('I will check.<|start|>assistant<|channel|>commentary to=functions.get_weather '
               '<|constrain|>json<|message|>{"location": "Seattle"}<|call|>')
    content, calls = parse_tool_calls(harmony, tools)
    assert content == "I will check." and calls[0]["function"]["name"] == "get_weather"
    assert json.loads(calls[0]["function"]["arguments"]) == {"location": "Seattle"}
    content, calls = parse_tool_calls('ok <tool_call>{"name": "get_weather", "arguments": {"q": 1}}</tool_call>', tools)
    assert content == "ok" and json.loads(calls[0]["function"]["arguments"]) == {"q": 1}
    content, calls = parse_tool_calls('{"name": "get_weather", "parameters": {"q": 2}}', tools)
    assert content is None and json.loads(calls[0]["function"]["arguments"]) == {"q": 2}
    content, calls = parse_tool_calls('{"name": "other", "arguments": {}}', tools)  # unknown tool: plain text
    assert calls == [] and content.startswith("{")
    assert parse_tool_calls("just text", tools) == ("just text", [])
