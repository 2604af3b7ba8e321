"""OpenAI-compatible HTTP server (``/v1/completions``, ``/v1/chat/completions``,
``/v1/models``, ``/health``, ``/metrics``, ``/start_profile``, ``/stop_profile``).

Request and response bodies follow the OpenAI / vLLM schema for the supported fields.
Prompts may be text (needs a tokenizer in the model directory) or token-id lists.
Profiling endpoints map to ``torch.profiler`` with CUDA activities (the Trainium
plugin mapped them to its device profiler, ``vllm/worker/neuron_profiler.py:52``).
"""

from __future__ import annotations

import asyncio
import json
import os
import time
import uuid

from fastapi import FastAPI, Request
from fastapi.responses import JSONResponse, PlainTextResponse, StreamingResponse

from ..engine.async_engine import AsyncLLM
from ..engine.sampling_params import SamplingParams
from ..logging_config import init_logger
from .tool_calls import ToolChoiceError, message_with_tools, tool_constraint, tools_prompt

logger = init_logger(__name__)


def _structured_from(body: dict) -> dict | None:
    """OpenAI ``response_format`` (json_object / json_schema) and vLLM's ``structured_outputs``
    / ``guided_json`` / ``guided_regex`` / ``guided_choice`` / ``guided_grammar`` fields."""
    if body.get("structured_outputs"):
        return dict(body["structured_outputs"])
    rf = body.get("response_format") or {}
    if rf.get("type") == "json_object":
        return {"json_object": True}
    if rf.get("type") == "json_schema":
        js = rf.get("json_schema") or {}
        return {"json": js.get("schema", js)}
    for key, field in (("guided_json", "json"), ("guided_regex", "regex"), ("guided_choice", "choice"),
                       ("guided_grammar", "grammar")):
        if body.get(key) is not None:
            return {field: body[key]}
    return None


def _sampling_from(body: dict) -> SamplingParams:
    return SamplingParams(
        temperature=float(body.get("temperature", 1.0)), top_p=float(body.get("top_p", 1.0)),
        top_k=int(body.get("top_k", 0) or 0), max_tokens=int(body.get("max_tokens", 16) or 16),
        min_tokens=int(body.get("min_tokens", 0) or 0), seed=body.get("seed"),
        stop_token_ids=body.get("stop_token_ids"), ignore_eos=bool(body.get("ignore_eos", False)),
        structured_outputs=_structured_from(body), logprobs=_logprobs_from(body), stop=body.get("stop"),
        n=int(body.get("n", 1) or 1),
        include_stop_str_in_output=bool(body.get("include_stop_str_in_output", False)))


def _logprobs_from(body: dict) -> int | None:
    """completions: ``logprobs: N``; chat: ``logprobs: true`` + ``top_logprobs: N``."""
    lp = body.get("logprobs")
    if lp is True:
        return int(body.get("top_logprobs") or 0)
    if lp is None or lp is False:
        return None
    return int(lp)


def _logprobs_payload(token_ids, entries, detok, chat: bool) -> dict | None:
    if entries is None:
        return None
    if chat:
        return {"content": [{"token": detok([t]), "logprob": e.get(t),
                             "top_logprobs": [{"token": detok([i]), "logprob": v} for i, v in e.items() if i != t]}
                            for t, e in zip(token_ids, entries)]}
    return {"tokens": [detok([t]) for t in token_ids], "token_logprobs": [e.get(t) for t, e in zip(token_ids, entries)],
            "top_logprobs": [{detok([i]): v for i, v in e.items()} for e in entries]}


def build_app(engine: AsyncLLM, served_name: str, tool_parser: str = "auto"):
    app = FastAPI(title="vllm_neuron_b200")
    state = {"prof": None}

    def tokenize(prompt):
        if isinstance(prompt, list) and prompt and isinstance(prompt[0], int):
            return prompt, None
        tok = engine.llm.get_tokenizer()
        return tok.encode(prompt), prompt

    def detok(ids):
        try:  # the end-of-sequence token (kept in token_ids) is not part of the text
            return engine.llm.get_tokenizer().decode(ids, skip_special_tokens=True)
        except Exception:  # noqa: BLE001
            return ""

    @app.get("/health")
    async def health():
        return {"status": "ok"}

    @app.get("/v1/models")
    async def models():
        return {"object": "list", "data": [{"id": served_name, "object": "model", "owned_by": "vllm_neuron_b200"}]}

    @app.get("/metrics")
    async def metrics():
        from prometheus_client import CONTENT_TYPE_LATEST, generate_latest

        return PlainTextResponse(generate_latest(), media_type=CONTENT_TYPE_LATEST)

    @app.post("/start_profile")
    async def start_profile():
        try:
            engine.call(lambda e: e.start_profile())
        except RuntimeError as e:
            return JSONResponse({"error": str(e)}, status_code=400)
        return {"status": "started"}

    @app.post("/stop_profile")
    async def stop_profile():
        try:
            res = engine.call(lambda e: e.stop_profile())
        except RuntimeError as e:
            return JSONResponse({"error": str(e)}, status_code=400)
        return {"status": "stopped", **res}

    async def _complete(ids, sp, stream: bool, chat: bool, rid: str, kvp: dict | None = None,
                        tools: tuple | None = None):
        """``tools``: (tools, tool_choice, parser) of a chat request that declared functions."""
        created = int(time.time())
        obj = "chat.completion" if chat else "text_completion"

        def choice(text, token_ids, finish):
            if chat:
                msg, called = {"role": "assistant", "content": text}, False
                if tools is not None:
                    msg, called = message_with_tools(text, *tools)
                return {"index": 0, "message": msg, "finish_reason": "tool_calls" if called else finish,
                        "token_ids": token_ids}
            return {"index": 0, "text": text, "finish_reason": finish, "token_ids": token_ids}

        if stream and sp.n > 1:
            return JSONResponse({"error": "n > 1 is not supported with stream=true"}, status_code=400)
        if stream and tools is not None:
            # tool calls are parsed from the whole generation: one delta with the message
            async def gen_tools():
                final = None
                async for o in engine.generate(ids, sp, rid, kv_transfer_params=kvp):
                    final = o
                c0 = final.outputs[0]
                ch = choice(c0.text if isinstance(c0.stop_reason, str) else detok(c0.token_ids), c0.token_ids,
                            c0.finish_reason)
                delta = {k: v for k, v in ch["message"].items() if v is not None}
                chunk = {"id": rid, "object": obj + ".chunk", "created": created, "model": served_name,
                         "choices": [{"index": 0, "delta": delta, "finish_reason": ch["finish_reason"],
                                      "token_ids": c0.token_ids}]}
                yield "data: " + json.dumps(chunk) + "\n\n"
                yield "data: [DONE]\n\n"

            return StreamingResponse(gen_tools(), media_type="text/event-stream")
        if stream:
            async def gen():
                sent = 0
                async for o in engine.generate(ids, sp, rid, kv_transfer_params=kvp):
                    toks = o.outputs[0].token_ids
                    new = toks[sent:]
                    sent = len(toks)
                    delta = detok(new)
                    ch = ({"index": 0, "delta": {"content": delta}, "finish_reason": o.outputs[0].finish_reason}
                          if chat else {"index": 0, "text": delta, "finish_reason": o.outputs[0].finish_reason})
                    ch["token_ids"] = new
                    chunk = {"id": rid, "object": obj + ".chunk", "created": created, "model": served_name,
                             "choices": [ch]}
                    if o.finished and o.kv_transfer_params is not None:
                        # disaggregated serving: the final chunk carries the transfer parameters
                        # (e.g. decode -> prefill KV of a multi-turn chat)
                        chunk["kv_transfer_params"] = o.kv_transfer_params
                    yield "data: " + json.dumps(chunk) + "\n\n"
                yield "data: [DONE]\n\n"

            return StreamingResponse(gen(), media_type="text/event-stream")
        if sp.n > 1:  # parallel sampling: n child requests, one choice each
            async def one(j):
                last = None
                async for o in engine.generate(ids, sp, f"{rid}#{j}", kv_transfer_params=kvp):
                    last = o
                return last

            finals = await asyncio.gather(*[one(j) for j in range(sp.n)])
            chs = []
            for j, f in enumerate(finals):
                c = f.outputs[0]
                ch = choice(c.text if isinstance(c.stop_reason, str) else detok(c.token_ids), c.token_ids,
                            c.finish_reason)
                ch["index"] = j
                ch["logprobs"] = _logprobs_payload(c.token_ids, c.logprobs, detok, chat)
                chs.append(ch)
            n_out = sum(len(f.outputs[0].token_ids) for f in finals)
            return {"id": rid, "object": obj, "created": created, "model": served_name, "choices": chs,
                    "usage": {"prompt_tokens": len(ids), "completion_tokens": n_out, "total_tokens": len(ids) + n_out}}
        final = None
        async for o in engine.generate(ids, sp, rid, kv_transfer_params=kvp):
            final = o
        toks = final.outputs[0].token_ids
        c0 = final.outputs[0]
        ch = choice(c0.text if isinstance(c0.stop_reason, str) else detok(toks), toks, c0.finish_reason)
        ch["logprobs"] = _logprobs_payload(toks, final.outputs[0].logprobs, detok, chat)
        resp = {"id": rid, "object": obj, "created": created, "model": served_name,
                "choices": [ch],
                "usage": {"prompt_tokens": len(ids), "completion_tokens": len(toks),
                          "total_tokens": len(ids) + len(toks)}}
        if final.kv_transfer_params is not None:
            resp["kv_transfer_params"] = final.kv_transfer_params
        return resp

    @app.exception_handler(ValueError)
    async def refused(_req: Request, e: ValueError):  # a request the engine refused (shape, grammar, ...)
        return JSONResponse({"error": str(e)}, status_code=400)

    @app.post("/v1/completions")
    async def completions(req: Request):
        body = await req.json()
        ids, _ = tokenize(body["prompt"])
        return await _complete(ids, _sampling_from(body), bool(body.get("stream", False)), False,
                               f"cmpl-{uuid.uuid4().hex}", body.get("kv_transfer_params"))

    @app.post("/v1/chat/completions")
    async def chat(req: Request):
        body = await req.json()
        msgs = body["messages"]
        tools = body.get("tools") or None
        tool_choice = body.get("tool_choice", "auto" if tools else None)
        if tool_choice == "none":
            tools = None
        try:
            constraint = tool_constraint(tools, tool_choice)
        except ToolChoiceError as e:
            return JSONResponse({"error": str(e)}, status_code=400)
        if constraint is not None:
            if _structured_from(body) is not None:
                return JSONResponse({"error": "tool_choice and response_format cannot be combined"},
                                    status_code=400)
            body = dict(body, structured_outputs=constraint)
        sp = _sampling_from(body)
        tok = engine.llm.get_tokenizer()
        if getattr(tok, "chat_template", None):
            ids = tok.apply_chat_template(msgs, tools=tools, add_generation_prompt=True, tokenize=True)
        else:
            head = tools_prompt(tools) + "\n" if tools else ""
            ids = tok.encode(head + "\n".join(f"{m['role']}: {m.get('content') or ''}" for m in msgs)
                             + "\nassistant:")
        spec = (tools, tool_choice, tool_parser) if tools else None
        return await _complete(list(ids), sp, bool(body.get("stream", False)), True,
                               f"chatcmpl-{uuid.uuid4().hex}", tools=spec)

    return app


def serve(engine_kwargs: dict, host: str = "127.0.0.1", port: int = 8000, served_name: str | None = None,
          tool_parser: str = "auto") -> None:
    import uvicorn

    engine = AsyncLLM(**engine_kwargs)
    name = served_name or str(engine_kwargs.get("model") or "model")
    app = build_app(engine, name, tool_parser)
    try:
        uvicorn.run(app, host=host, port=port, log_level="warning")
    finally:
        engine.shutdown()
