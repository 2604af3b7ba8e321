"""Toy router for disaggregated serving (1 prefill server, 1 decode server), the counterpart of
the Trainium plugin's ``examples/vllm_neuron/vllm/disaggregated_inference/toy_proxy_server.py``.

For every ``/v1/completions`` request it
1. sends the prompt to the prefill server with ``max_tokens=1`` and
   ``kv_transfer_params={"do_remote_decode": True}`` (the prefill engine exports the prompt KV);
2. forwards the original request to the decode server with the ``kv_transfer_params`` the
   prefill server returned (the decode engine loads the KV and generates), streaming or not.

Multi-turn chats with bidirectional KV (``VLLM_B200_BIDIRECTIONAL_KV=1`` on both servers, the
prefill server in ``kv_role: kv_both``): a request whose ``kv_transfer_params`` carry
``"return_kv": true`` (the client expects another turn) makes the decode server export the
conversation when it finishes, and its (non-streaming) response carries ``kv_transfer_params``
for it; a client that sends them back with the next turn's request makes the prefill server
load that prefix from the decode server instead of recomputing it (the reference proxy relays
the decode side's block ids the same way).  Requests without the flag export nothing.

``vllm-b200 disagg-proxy --prefill http://127.0.0.1:8100 --decode http://127.0.0.1:8200 --port 8000``
"""

from __future__ import annotations

from typing import Awaitable, Callable

from fastapi import FastAPI, Request
from fastapi.responses import JSONResponse, StreamingResponse

PostFn = Callable[[str, dict], Awaitable[dict]]


async def _aiohttp_post(url: str, body: dict) -> dict:
    import aiohttp

    async with aiohttp.ClientSession() as s:
        async with s.post(url, json=body) as r:
            r.raise_for_status()
            return await r.json()


def build_proxy(prefill_url: str, decode_url: str, post: PostFn | None = None) -> FastAPI:
    app = FastAPI()
    post = post or _aiohttp_post
    stats = {"requests": 0, "transfers": 0}

    async def _prefill(body: dict) -> dict:
        prev = body.get("kv_transfer_params") or {}  # a previous turn's decode -> prefill transfer
        pb = dict(body, max_tokens=1, stream=False, kv_transfer_params={**prev, "do_remote_decode": True})
        resp = await post(prefill_url.rstrip("/") + "/v1/completions", pb)
        kvp = resp.get("kv_transfer_params")
        if not kvp:
            raise RuntimeError("prefill server returned no kv_transfer_params (is it a kv_producer?)")
        stats["transfers"] += 1
        return kvp

    @app.get("/health")
    async def health():
        return {"status": "ok", **stats}

    @app.post("/v1/completions")
    async def completions(req: Request):
        body = await req.json()
        stats["requests"] += 1
        try:
            kvp = await _prefill(body)
        except Exception as e:  # noqa: BLE001
            return JSONResponse({"error": f"prefill failed: {e}"}, status_code=502)
        wants_kv_back = bool((body.get("kv_transfer_params") or {}).get("return_kv"))
        db = dict(body, kv_transfer_params={**kvp, "return_kv": True} if wants_kv_back else kvp)
        if body.get("stream"):
            import aiohttp

            async def gen():
                async with aiohttp.ClientSession() as s:
                    async with s.post(decode_url.rstrip("/") + "/v1/completions", json=db) as r:
                        async for chunk in r.content.iter_any():
                            yield chunk

            return StreamingResponse(gen(), media_type="text/event-stream")
        resp = await post(decode_url.rstrip("/") + "/v1/completions", db)
        return JSONResponse(resp)

    return app


def serve_proxy(prefill_url: str, decode_url: str, host: str = "127.0.0.1", port: int = 8000) -> None:
    import uvicorn

    uvicorn.run(build_proxy(prefill_url, decode_url), host=host, port=port, log_level="warning")


if __name__ == "__main__":  # pragma: no cover
    import argparse

    ap = argparse.ArgumentParser()
    ap.add_argument("--prefill", required=True)
    ap.add_argument("--decode", required=True)
    ap.add_argument("--port", type=int, default=8000)
    a = ap.parse_args()
    serve_proxy(a.prefill, a.decode, port=a.port)
