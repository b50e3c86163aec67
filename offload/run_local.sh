#!/usr/bin/env bash
# Local experiment: server and mobile client on this host over loopback TCP.
#   bash offload/run_local.sh offload/config/<exp>.json [extra mobile args, e.g. -nr 20 --set k=v]
# Server options come from SERVER_ARGS (e.g. SERVER_ARGS="--tp 2 --device cuda:0").
set -euo pipefail
CFG="${1:?usage: run_local.sh CONFIG.json [mobile args]}"
shift
ROOT="$(cd "$(dirname "${BASH_SOURCE[0]}")/.." && pwd)"
export PYTHONPATH="$ROOT${PYTHONPATH:+:$PYTHONPATH}"
python -m offload.server.main --listen-host 127.0.0.1 ${SERVER_ARGS:-} &
SRV=$!
trap 'kill $SRV 2>/dev/null || true; wait $SRV 2>/dev/null || true' EXIT
sleep 3
python -m offload.mobile.main --ip 127.0.0.1 --config "$CFG" "$@"
