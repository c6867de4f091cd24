#!/usr/bin/env bash
# Coordinator container: wait for the object store, create checkpoint v0 if the store has none, then
# run the HTTP coordinator in the foreground. Storage and coordinator knobs come from the environment
# (R2_ENDPOINT, R2_BUCKET, R2_ACCESS_KEY_ID, R2_SECRET_ACCESS_KEY, R2_REGION, PORT, HOST,
# MIN_CONTRIBUTIONS, OUTER_LR, OUTER_MOMENTUM, KEEP_VERSIONS, MAX_STALENESS, VOCAB_SIZE, MIN_WEIGHT,
# STALENESS_DECAY, S3_EXTERNAL_ENDPOINT); PRESET / SEED choose the bootstrap model.
# DT_DRY_RUN=1 prints the commands instead of running them.
set -euo pipefail

PRESET="${PRESET:-tiny}"
SEED="${SEED:-0}"
PORT="${PORT:-8000}"
MERGE_DEVICE="${MERGE_DEVICE:-cpu}"
STORE_WAIT_SECS="${STORE_WAIT_SECS:-60}"
PY="${PYTHON:-python}"
export PORT

run() {
    if [ "${DT_DRY_RUN:-0}" = "1" ]; then echo "$*"; else "$@"; fi
}

if [ -n "${R2_ENDPOINT:-}" ] && [ "${DT_DRY_RUN:-0}" != "1" ]; then
    echo "[coordinator] waiting for object store ${R2_ENDPOINT} (up to ${STORE_WAIT_SECS}s)"
    ok=0
    for _ in $(seq 1 "${STORE_WAIT_SECS}"); do
        if curl -s -o /dev/null --max-time 2 "${R2_ENDPOINT}"; then ok=1; break; fi
        sleep 1
    done
    if [ "$ok" != "1" ]; then echo "[coordinator] object store not reachable" >&2; exit 1; fi
fi
if [ -z "${S3_EXTERNAL_ENDPOINT:-}" ]; then
    echo "[coordinator] S3_EXTERNAL_ENDPOINT not set: nodes outside this host get ${R2_ENDPOINT:-the default endpoint} from /config"
fi

run "$PY" -m distrain_b200 bootstrap --if-absent --preset "$PRESET" --seed "$SEED"
run exec "$PY" -m distrain_b200 coordinator --port "$PORT" --merge-device "$MERGE_DEVICE"
