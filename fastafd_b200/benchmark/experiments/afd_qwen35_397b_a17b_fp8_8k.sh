#!/usr/bin/env bash
# Qwen3.5-397B-A17B-FP8 (gated DeltaNet + gated attention hybrid), 8K context.
source "$(dirname "${BASH_SOURCE[0]}")/common.sh"
export PRESET_NAME="afd_qwen35_397b_a17b_fp8_8k"
export MODEL="${MODEL:-qwen3.5-397b-a17b-fp8}"
export PROMPT_LEN="${PROMPT_LEN:-8192}"
export PER_ATTN_GPU_BSZ="${PER_ATTN_GPU_BSZ:-128}"
export NUM_GPUS="${NUM_GPUS:-8}"
export ATTN_GPUS="${ATTN_GPUS:-4}"
export STEPS="${STEPS:-32}"
export ATTN_TP="${ATTN_TP:-1}"     # attention data-parallel lanes (ATTN_TP=4: one tensor-parallel lane)
fastafd_run_bench
