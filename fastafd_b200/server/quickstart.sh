#!/usr/bin/env bash
# Quick start on one machine: build the kernels, check alignment against the PyTorch oracle,
# start a server for the tiny random-weight model and send it one request.
#   ./quickstart.sh            # GPU 0 if there is one, else CPU
#   DEVICE=cpu ./quickstart.sh
# Reference: scripts/quickstart (one-command bring-up of a small model).
set -euo pipefail
cd "$(dirname "$0")/../.."
PORT="${PORT:-1919}"
DEVICE="${DEVICE:-$(python -c 'import torch; print("cuda:0" if torch.cuda.is_available() else "cpu")')}"

echo "== build"
python -m fastafd_b200.build
echo "== alignment against the PyTorch oracle ($DEVICE)"
python -m fastafd_b200.validate --model tiny-qwen3-moe --device "$DEVICE" --prompts 4 --prompt-len 32 --decode 16

echo "== server on port $PORT"
python -m fastafd_b200 --mode afd-serve --model-path tiny-qwen3-moe --device "${DEVICE%%:*}" --host 127.0.0.1 \
  --port "$PORT" --afd-num-mb 2 --num-pages 64 --max-seq-len-override 128 --afd-max-running-requests 8 \
  --cuda-graph-max-bs 8 &
SERVER=$!
trap 'kill $SERVER 2>/dev/null || true' EXIT
for _ in $(seq 1 120); do
  if curl -sf "http://127.0.0.1:$PORT/v1/models" > /dev/null; then break; fi
  sleep 1
done
echo "== one request"
curl -sf "http://127.0.0.1:$PORT/v1/chat/completions" -H 'content-type: application/json' \
  -d '{"input_ids": [1, 2, 3, 4, 5, 6, 7, 8], "max_tokens": 8, "ignore_eos": true, "stream": false, "return_token_ids": true}'
echo
