"""``vllm-b200`` command line: ``serve`` (OpenAI server) and ``bench`` (serving benchmark
client with random prompts).  Flags use vLLM's names so launch scripts carry over, e.g.::

    vllm-b200 serve /models/gpt-oss-120b --tensor-parallel-size 8 --max-model-len 8192 \\
        --max-num-seqs 64 --max-num-batched-tokens 4096 --block-size 32 \\
        --additional-config '{"neuron_config": {"ep_degree": 8}}'
"""

from __future__ import annotations

import argparse
import json


def _engine_args(ap: argparse.ArgumentParser) -> None:
    ap.add_argument("model", nargs="?", default=None)
    ap.add_argument("--tensor-parallel-size", "-tp", type=int, default=1)
    ap.add_argument("--data-parallel-size", "-dp", type=int, default=1)
    ap.add_argument("--enable-expert-parallel", action="store_true")
    ap.add_argument("--decode-context-parallel-size", "-dcp", type=int, default=1)
    ap.add_argument("--all2all-backend", default="allgather_reducescatter",
                    choices=["allgather_reducescatter", "naive", "neuron", "b200"],
                    help="MoE token exchange under data parallelism (neuron / b200: fused NVLink all-to-all)")
    ap.add_argument("--max-model-len", type=int, default=8192)
    ap.add_argument("--max-num-seqs", type=int, default=64)
    ap.add_argument("--max-num-batched-tokens", type=int, default=4096)
    ap.add_argument("--block-size", type=int, default=32)
    ap.add_argument("--kv-cache-dtype", default="auto")
    ap.add_argument("--gpu-memory-utilization", type=float, default=0.9)
    ap.add_argument("--enable-prefix-caching", action="store_true")
    ap.add_argument("--enforce-eager", action="store_true")
    ap.add_argument("--async-scheduling", action="store_true",
                    help="stage decode step k+1 on the host while step k runs on the GPU")
    ap.add_argument("--load-format", default="auto")
    ap.add_argument("--dtype", default="bfloat16")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--speculative-config", type=json.loads, default=None)
    ap.add_argument("--kv-transfer-config", type=json.loads, default=None)
    ap.add_argument("--additional-config", type=json.loads, default=None)
    ap.add_argument("--hf-config", type=json.loads, default=None, help="config.json contents (dummy weights)")
    ap.add_argument("--served-model-name", default=None)


def engine_kwargs(a) -> dict:
    kw = dict(model=a.model, tensor_parallel_size=a.tensor_parallel_size, data_parallel_size=a.data_parallel_size,
              max_model_len=a.max_model_len, max_num_seqs=a.max_num_seqs,
              max_num_batched_tokens=a.max_num_batched_tokens, block_size=a.block_size,
              kv_cache_dtype=a.kv_cache_dtype, gpu_memory_utilization=a.gpu_memory_utilization,
              enable_prefix_caching=a.enable_prefix_caching, enforce_eager=a.enforce_eager,
              load_format=a.load_format, dtype=a.dtype, seed=a.seed, speculative_config=a.speculative_config,
              kv_transfer_config=a.kv_transfer_config, additional_config=a.additional_config,
              served_model_name=a.served_model_name, enable_expert_parallel=a.enable_expert_parallel,
              async_scheduling=a.async_scheduling, decode_context_parallel_size=a.decode_context_parallel_size,
              all2all_backend=a.all2all_backend)
    if a.hf_config is not None:
        kw["hf_config"] = a.hf_config
        kw["load_format"] = "dummy"
    return kw


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(prog="vllm-b200")
    sub = ap.add_subparsers(dest="cmd", required=True)
    s = sub.add_parser("serve", help="OpenAI-compatible server")
    _engine_args(s)
    s.add_argument("--host", default="127.0.0.1")
    s.add_argument("--port", type=int, default=8000)
    s.add_argument("--tool-call-parser", default="auto", choices=["auto", "openai", "hermes", "json"],
                   help="how tool calls are read from text when tool_choice is auto")
    s.add_argument("--enable-auto-tool-choice", action="store_true",
                   help="accepted for compatibility (auto tool choice is always available)")
    b = sub.add_parser("bench", help="serving benchmark client (random prompts)")
    b.add_argument("--base-url", default="http://127.0.0.1:8000")
    b.add_argument("--num-prompts", type=int, default=64)
    b.add_argument("--max-concurrency", type=int, default=64)
    b.add_argument("--random-input-len", type=int, default=1024)
    b.add_argument("--random-output-len", type=int, default=128)
    b.add_argument("--vocab", type=int, default=32000)
    x = sub.add_parser("disagg-proxy", help="router for one prefill and one decode server")
    x.add_argument("--prefill", required=True, help="prefill server base URL (kv_producer)")
    x.add_argument("--decode", required=True, help="decode server base URL (kv_consumer)")
    x.add_argument("--host", default="127.0.0.1")
    x.add_argument("--port", type=int, default=8000)
    a = ap.parse_args(argv)
    if a.cmd == "disagg-proxy":
        from .disagg_proxy import serve_proxy

        serve_proxy(a.prefill, a.decode, a.host, a.port)
    elif a.cmd == "serve":
        from .openai_server import serve

        serve(engine_kwargs(a), a.host, a.port, a.served_model_name, a.tool_call_parser)
    else:
        from .bench_client import run_bench

        print(json.dumps(run_bench(a)))


if __name__ == "__main__":
    main()
