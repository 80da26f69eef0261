#!/usr/bin/env bash
# Start an AFD server on one machine. Defaults: 8 GPUs = 4 attention GPUs (data-parallel lanes) + 4 expert
# GPUs (expert parallel), two micro-batches, three steps planned ahead.
#
#   fastafd_server.sh --model PATH [--host H] [--port P] [any flag of `python -m fastafd_b200`] [--extra-args "..."]
#   MODEL=/path/to/checkpoint-or-preset PORT=1919 ./fastafd_server.sh [flags]
#
# Every flag of the reference's serve script is accepted under its name (they are flags of the CLI
# here: --launch-backend, --ray-*, --afd-*-size, --afd-num-mb, --cache-type, --cuda-graph-max-bs, ...);
# a flag given on the command line overrides the default below. --env NAME checks the active conda
# environment like the reference's script does, --extra-args appends shell words.
# Reference: scripts/serve/fastafd_server.sh:9-43,144-198.
set -euo pipefail

usage() { sed -n '2,12p' "$0" | sed 's/^# \{0,1\}//'; }

MODEL="${MODEL:-qwen3-30b-a3b}"
HOST="${HOST:-0.0.0.0}"
PORT="${PORT:-1919}"
ENV_NAME=""
EXTRA_ARGS=""
PASS=()
while [[ $# -gt 0 ]]; do
  case "$1" in
    -h|--help) usage; exit 0 ;;
    --model|--model-path) MODEL="$2"; shift 2 ;;
    --host) HOST="$2"; shift 2 ;;
    --port) PORT="$2"; shift 2 ;;
    --env) ENV_NAME="$2"; shift 2 ;;
    --extra-args) EXTRA_ARGS="$2"; shift 2 ;;
    *) PASS+=("$1"); shift ;;
  esac
done
if [[ -n "$ENV_NAME" && "${CONDA_DEFAULT_ENV:-}" != "$ENV_NAME" ]]; then
  echo "expected conda env '$ENV_NAME', active: '${CONDA_DEFAULT_ENV:-none}'" >&2
  exit 2
fi

# defaults that a flag among the passed ones replaces (argparse keeps the last occurrence)
DEFAULTS=(--afd-attn-dp-size "${ATTN_DP:-4}" --afd-attn-tp-size "${ATTN_TP:-1}" --afd-mlp-ep-size "${MLP_EP:-4}"
          --afd-num-mb "${NUM_MB:-2}" --afd-async-pending-steps 3 --page-size 16 --cache-type naive)
# shellcheck disable=SC2206
EXTRA=($EXTRA_ARGS)
CMD=(python -m fastafd_b200 --mode afd-serve --model-path "$MODEL" --host "$HOST" --port "$PORT"
     "${DEFAULTS[@]}" "${PASS[@]}" "${EXTRA[@]}")
if [[ "${DRY_RUN:-0}" == "1" ]]; then printf '%s\n' "${CMD[*]}"; exit 0; fi
exec "${CMD[@]}"
