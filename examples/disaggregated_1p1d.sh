#!/usr/bin/env bash
# Disaggregated prefill / decode on one 8-GPU host: a prefill server on GPUs 0-3 (kv_producer),
# a decode server on GPUs 4-7 (kv_consumer) and the router in front.  The KV of each prompt
# moves through the shared store directory (byte-exact; producer and consumer may use
# different TP degrees).
set -euo pipefail
MODEL=${1:-/models/gpt-oss-120b}
STORE=/dev/shm/b200_kv_store
mkdir -p "$STORE"
KV_P='{"kv_connector": "HostStagedConnector", "kv_role": "kv_producer", "kv_connector_extra_config": {"store_path": "'$STORE'"}}'
KV_D='{"kv_connector": "HostStagedConnector", "kv_role": "kv_consumer", "kv_connector_extra_config": {"store_path": "'$STORE'"}}'
CUDA_VISIBLE_DEVICES=0,1,2,3 vllm-b200 serve "$MODEL" -tp 4 --port 8100 --kv-transfer-config "$KV_P" &
P=$!
CUDA_VISIBLE_DEVICES=4,5,6,7 vllm-b200 serve "$MODEL" -tp 4 --port 8200 --kv-transfer-config "$KV_D" &
D=$!
trap 'kill $P $D' EXIT
for port in 8100 8200; do until curl -sf http://127.0.0.1:$port/health >/dev/null; do sleep 5; done; done
vllm-b200 disagg-proxy --prefill http://127.0.0.1:8100 --decode http://127.0.0.1:8200 --port 8000
