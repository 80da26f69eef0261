#!/usr/bin/env bash
# Shared part of the experiment presets: every preset sets a workload through environment variables
# (each one keeps a value that the caller exported) and calls fastafd_run_bench, which launches
# bench.py with one process per GPU, keeps stdout/stderr and the JSON line in a run directory and,
# when SUITE_NAME names an entry of benchmark/configs.json, checks the step time against the value
# recorded there (+-3 % by default).
#   MODEL PROMPT_LEN PER_ATTN_GPU_BSZ NUM_GPUS ATTN_GPUS ATTN_TP NUM_MB STEPS WARMUP SPEC_BLOCK
#   SPEC_ACCEPT ROUTER_BIAS RUN_DIR MASTER_PORT TP_FUSED DRY_RUN
# Reference: scripts/lib/common.sh and scripts/experiments/afd/*/run_*.sh (workload shape per preset,
# thin wrappers around one runner).
set -euo pipefail

fastafd_repo_root() {
  local d
  d="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
  while [[ "$d" != "/" && ! -f "$d/bench.py" ]]; do d="$(dirname "$d")"; done
  [[ -f "$d/bench.py" ]] || { echo "bench.py not found above ${BASH_SOURCE[0]}" >&2; return 1; }
  echo "$d"
}

fastafd_run_bench() {
  local root ts run_dir
  root="$(fastafd_repo_root)"
  ts="$(date -u +%Y%m%d_%H%M%S)"
  : "${MODEL:?MODEL is not set}" "${PROMPT_LEN:?}" "${PER_ATTN_GPU_BSZ:?}"
  local gpus="${NUM_GPUS:-8}" steps="${STEPS:-64}" warmup="${WARMUP:-8}"
  run_dir="${RUN_DIR:-$root/benchmark-runs/${PRESET_NAME:-run}_${gpus}gpu_b${PER_ATTN_GPU_BSZ}_${ts}}"
  mkdir -p "$run_dir"
  local args=(bench.py --gpus "$gpus" --steps "$steps" --warmup "$warmup" --model "$MODEL"
              --batch-per-attn-gpu "$PER_ATTN_GPU_BSZ" --context "$PROMPT_LEN")
  [[ -n "${NUM_MB:-}" ]] && args+=(--num-mb "$NUM_MB")
  [[ -n "${ATTN_GPUS:-}" && "$gpus" -gt 1 ]] && args+=(--attn-gpus "$ATTN_GPUS")
  [[ -n "${ATTN_TP:-}" && "$gpus" -gt 1 ]] && args+=(--attn-tp "$ATTN_TP")
  [[ -n "${SPEC_BLOCK:-}" ]] && args+=(--spec-block "$SPEC_BLOCK" --spec-sim-accept "${SPEC_ACCEPT:-1.8}")
  [[ -n "${ROUTER_BIAS:-}" ]] && args+=(--also-router-bias "$ROUTER_BIAS")
  [[ -n "${TP_FUSED:-}" ]] && export FASTAFD_TP_FUSED="$TP_FUSED"
  local cmd
  if [[ "$gpus" -gt 1 ]]; then
    cmd=(python -m torch.distributed.run --nnodes=1 --nproc-per-node "$gpus" --master-addr 127.0.0.1
         --master-port "${MASTER_PORT:-29541}" "${args[@]}")
  else
    cmd=(python "${args[@]}")
  fi
  printf '%s\n' "${cmd[*]}" > "$run_dir/command.txt"
  echo "== ${PRESET_NAME:-run}: ${cmd[*]}"
  if [[ "${DRY_RUN:-0}" == "1" ]]; then return 0; fi      # print the command, run nothing
  (cd "$root" && "${cmd[@]}") > "$run_dir/stdout.log" 2> "$run_dir/stderr.log" || {
    echo "bench failed; see $run_dir/stderr.log" >&2; tail -5 "$run_dir/stderr.log" >&2; return 1; }
  grep '"metric"' "$run_dir/stdout.log" | tail -1 > "$run_dir/bench.json"
  cat "$run_dir/bench.json"
  if [[ -n "${SUITE_NAME:-}" ]]; then
    (cd "$root" && python - "$SUITE_NAME" "$run_dir/bench.json" <<'PY'
import json, sys
from fastafd_b200.benchmark import suite
cfgs = suite.load_configs()
c = cfgs["configs"][sys.argv[1]]
res = suite.evaluate(c, open(sys.argv[2]).read().strip(), c.get("tolerance", cfgs.get("tolerance", 0.03)))
print(json.dumps(res))
PY
    ) | tee "$run_dir/result.json"
  fi
  echo "== run directory: $run_dir"
}
