#!/usr/bin/env bash
# Disaggregated prefill / decode on one 8-GPU host: a prefill server on GPUs 0-3 (kv_producer),
# a decode server on GPUs 4-7 (kv_consumer) and the router in front.  The KV of each prompt
# moves GPU to GPU: the prefill ranks gather it into a CUDA-IPC device pool and the decode
# ranks copy their kv heads straight into their blocks (B200IpcConnector; producer and
# consumer may use different TP degrees).  CUDA IPC maps only memory of GPUs the process can
# see, so both servers see all eight GPUs and the decode server starts at GPU 4
# (VLLM_B200_DEVICE_OFFSET).  TRANSPORT=HostStagedConnector moves the KV through files in the
# store directory instead.
set -euo pipefail
MODEL=${1:-/models/gpt-oss-120b}
STORE=/dev/shm/b200_kv_store
mkdir -p "$STORE"
TRANSPORT=${TRANSPORT:-B200IpcConnector}
KV_P='{"kv_connector": "'$TRANSPORT'", "kv_role": "kv_producer", "kv_connector_extra_config": {"store_path": "'$STORE'", "pool_mb": 4096}}'
KV_D='{"kv_connector": "'$TRANSPORT'", "kv_role": "kv_consumer", "kv_connector_extra_config": {"store_path": "'$STORE'"}}'
VLLM_B200_DEVICE_OFFSET=0 vllm-b200 serve "$MODEL" -tp 4 --port 8100 --kv-transfer-config "$KV_P" &
P=$!
VLLM_B200_DEVICE_OFFSET=4 vllm-b200 serve "$MODEL" -tp 4 --port 8200 --kv-transfer-config "$KV_D" &
D=$!
trap 'kill $P $D' EXIT
for port in 8100 8200; do until curl -sf http://127.0.0.1:$port/health >/dev/null; do sleep 5; done; done
vllm-b200 disagg-proxy --prefill http://127.0.0.1:8100 --decode http://127.0.0.1:8200 --port 8000
