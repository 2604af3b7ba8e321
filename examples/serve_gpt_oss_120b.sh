#!/usr/bin/env bash
# OpenAI-compatible server for GPT-OSS-120B (MXFP4 experts) on 8 B200s: attention TP=8,
# experts EP=8 over the same ranks, decode CUDA graphs for up to 64 sequences.
set -euo pipefail
MODEL=${1:-/models/gpt-oss-120b}
vllm-b200 serve "$MODEL" \
  --tensor-parallel-size 8 --enable-expert-parallel \
  --max-model-len 8192 --max-num-seqs 64 --max-num-batched-tokens 8192 --block-size 32 \
  --enable-prefix-caching \
  --additional-config '{"neuron_config": {"ep_degree": 8, "num_seqs_buckets": [1, 8, 16, 32, 64]}}' \
  --port 8000 &
SERVER=$!
trap 'kill $SERVER' EXIT
until curl -sf http://127.0.0.1:8000/health >/dev/null; do sleep 5; done
# random-prompt serving benchmark (2048 in / 512 out, 64 concurrent)
vllm-b200 bench --base-url http://127.0.0.1:8000 --num-prompts 256 --max-concurrency 64 \
  --random-input-len 2048 --random-output-len 512 --vocab 200000
