#!/usr/bin/env bash
# Start an AFD server on one 8-GPU machine: 4 attention GPUs (data parallel) + 4 expert GPUs
# (expert parallel), two micro-batches, three steps planned ahead.
# Usage: MODEL=/path/to/checkpoint-or-preset PORT=1919 ./fastafd_server.sh [extra flags]
set -euo pipefail
MODEL="${MODEL:-qwen3-30b-a3b}"
PORT="${PORT:-1919}"
ATTN_DP="${ATTN_DP:-4}"
ATTN_TP="${ATTN_TP:-1}"
MLP_EP="${MLP_EP:-4}"
NUM_MB="${NUM_MB:-2}"
exec python -m fastafd_b200 --mode afd-serve --model-path "$MODEL" --host 0.0.0.0 --port "$PORT" \
  --afd-attn-dp-size "$ATTN_DP" --afd-attn-tp-size "$ATTN_TP" --afd-mlp-ep-size "$MLP_EP" \
  --afd-num-mb "$NUM_MB" --afd-async-pending-steps 3 --page-size 16 --cache-type naive "$@"
