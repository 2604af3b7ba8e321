"""Serving benchmark client: random-token prompts at a fixed concurrency against the
OpenAI server, reporting output tok/s and p50 TTFT / TPOT (the metrics of
``vllm bench serve --dataset-name random``)."""

from __future__ import annotations

import asyncio
import json
import random
import statistics
import time


async def _one(session, url, prompt, out_len, stats):
    body = {"prompt": prompt, "max_tokens": out_len, "temperature": 0.0, "ignore_eos": True, "stream": True}
    t0 = time.perf_counter()
    first = None
    last = t0
    gaps = []
    n = 0
    async with session.post(url + "/v1/completions", json=body) as r:
        async for line in r.content:
            line = line.decode().strip()
            if not line.startswith("data:") or line.endswith("[DONE]"):
                continue
            now = time.perf_counter()
            ch = json.loads(line[5:])["choices"][0]
            k = len(ch.get("token_ids", [])) or 1
            if first is None:
                first = now
            else:
                gaps.append((now - last) / k)
            last = now
            n += k
    stats.append({"ttft": (first or last) - t0, "tpot": statistics.mean(gaps) if gaps else 0.0, "tokens": n})


async def _run(args):
    import aiohttp

    rng = random.Random(0)
    prompts = [[rng.randrange(10, args.vocab) for _ in range(args.random_input_len)] for _ in range(args.num_prompts)]
    stats: list = []
    sem = asyncio.Semaphore(args.max_concurrency)
    t0 = time.perf_counter()
    async with aiohttp.ClientSession(timeout=aiohttp.ClientTimeout(total=None)) as s:
        async def task(p):
            async with sem:
                await _one(s, args.base_url, p, args.random_output_len, stats)

        await asyncio.gather(*(task(p) for p in prompts))
    dur = time.perf_counter() - t0
    toks = sum(x["tokens"] for x in stats)
    return {"output_tok_s": toks / dur, "duration_s": dur, "completed": len(stats),
            "p50_ttft_ms": 1000 * statistics.median(x["ttft"] for x in stats),
            "p50_tpot_ms": 1000 * statistics.median(x["tpot"] for x in stats)}


def run_bench(args) -> dict:
    return asyncio.run(_run(args))
