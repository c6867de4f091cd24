#!/usr/bin/env bash
# HTTP node container: write node.toml from the environment (the reference node's config file:
# coordinator_url, gpu_device, inner-step bounds, push interval, cache, [storage]) and start a node on it.
# COORDINATOR_URL, S3_ENDPOINT, S3_BUCKET, S3_ACCESS_KEY, S3_SECRET_KEY, S3_REGION, GPU_DEVICE,
# MIN_INNER_STEPS, MAX_INNER_STEPS, PUSH_INTERVAL, BATCH_SIZE (optional), SEQ_LEN, CACHE_DIR, STEPS,
# DATA_DIR (optional local shards), NODE_ID (optional). DT_DRY_RUN=1 prints the file and the command only.
set -euo pipefail

CONFIG="${NODE_CONFIG:-/tmp/node.toml}"
CACHE_DIR="${CACHE_DIR:-/workspace/cache}"
PY="${PYTHON:-python}"

{
    echo "coordinator_url = \"${COORDINATOR_URL:-http://localhost:8000}\""
    echo "api_key = \"\""
    echo "gpu_device = ${GPU_DEVICE:-0}"
    echo "target_push_interval_secs = ${PUSH_INTERVAL:-60.0}"
    echo "min_inner_steps = ${MIN_INNER_STEPS:-50}"
    echo "max_inner_steps = ${MAX_INNER_STEPS:-500}"
    echo "cache_dir = \"${CACHE_DIR}\""
    echo "max_cache_gb = ${MAX_CACHE_GB:-100}"
    echo "seq_len = ${SEQ_LEN:-512}"
    if [ -n "${BATCH_SIZE:-}" ]; then echo "force_batch_size = ${BATCH_SIZE}"; fi
    echo ""
    echo "[storage]"
    echo "endpoint = \"${S3_ENDPOINT:-http://localhost:9000}\""
    echo "bucket = \"${S3_BUCKET:-distrain-training}\""
    echo "access_key_id = \"${S3_ACCESS_KEY:-minioadmin}\""
    echo "secret_access_key = \"${S3_SECRET_KEY:-minioadmin}\""
    echo "region = \"${S3_REGION:-us-east-1}\""
} > "$CONFIG"
echo "[node] wrote $CONFIG"

args=(-m distrain_b200 start --config "$CONFIG" --steps "${STEPS:-100000}")
if [ -n "${DATA_DIR:-}" ]; then args+=(--data-dir "$DATA_DIR"); fi
if [ -n "${NODE_ID:-}" ]; then args+=(--node-id "$NODE_ID"); fi
if [ "${DT_DRY_RUN:-0}" = "1" ]; then cat "$CONFIG"; echo "$PY ${args[*]}"; exit 0; fi
exec "$PY" "${args[@]}"
