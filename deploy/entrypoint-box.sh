#!/usr/bin/env bash
# In-box job container: every visible GPU is one node of the in-box protocol (compressed deltas over
# NVLink, distributed merge, NVLS broadcast), launched with torch.distributed.run on 127.0.0.1.
# PRESET, GPUS (default: all visible), STEPS, DATA_DIR, CHECKPOINT_STORE, CHECKPOINT_EVERY, RESUME=1,
# METRICS_PORT, PUSH_EVERY, LOG (JSONL path), MASTER_PORT, JOB_TIMEOUT_SECS (outer bound on the job).
# DT_DRY_RUN=1 prints the command only.
set -euo pipefail

PY="${PYTHON:-python}"
if [ -z "${GPUS:-}" ]; then
    GPUS=$(nvidia-smi --query-gpu=index --format=csv,noheader 2>/dev/null | wc -l || true)
    GPUS=${GPUS:-1}
    if [ "$GPUS" -lt 1 ]; then GPUS=1; fi
fi
args=(-m torch.distributed.run --nnodes 1 --nproc-per-node "$GPUS" --master-addr 127.0.0.1
      --master-port "${MASTER_PORT:-29511}" -m distrain_b200 train-box --preset "${PRESET:-tiny}"
      --steps "${STEPS:-100000}" --log-every "${LOG_EVERY:-50}")
if [ -n "${DATA_DIR:-}" ]; then args+=(--data-dir "$DATA_DIR"); fi
if [ -n "${CHECKPOINT_STORE:-}" ]; then args+=(--checkpoint-store "$CHECKPOINT_STORE" --checkpoint-every "${CHECKPOINT_EVERY:-10}"); fi
if [ "${RESUME:-0}" = "1" ]; then args+=(--resume); fi
if [ -n "${METRICS_PORT:-}" ]; then args+=(--metrics-port "$METRICS_PORT"); fi
if [ -n "${PUSH_EVERY:-}" ]; then args+=(--push-every "$PUSH_EVERY"); fi
if [ -n "${LOG:-}" ]; then args+=(--output "$LOG"); fi
if [ "${DT_DRY_RUN:-0}" = "1" ]; then echo "$PY ${args[*]}"; exit 0; fi
exec timeout -k 60 "${JOB_TIMEOUT_SECS:-31536000}" "$PY" "${args[@]}"
