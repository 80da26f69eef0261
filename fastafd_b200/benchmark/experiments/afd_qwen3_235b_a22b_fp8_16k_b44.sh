#!/usr/bin/env bash
# Qwen3-235B-A22B-FP8 decode replay, 16K context: twice the KV per request of the 8K preset, so half the batch.
source "$(dirname "${BASH_SOURCE[0]}")/common.sh"
export PRESET_NAME="afd_qwen3_235b_a22b_fp8_16k_b44"
export MODEL="${MODEL:-qwen3-235b-a22b-fp8}"
export PROMPT_LEN="${PROMPT_LEN:-16384}"
export PER_ATTN_GPU_BSZ="${PER_ATTN_GPU_BSZ:-44}"
export NUM_GPUS="${NUM_GPUS:-8}"
export ATTN_GPUS="${ATTN_GPUS:-4}"
export NUM_MB="${NUM_MB:-2}"
export STEPS="${STEPS:-32}"
export ATTN_TP="${ATTN_TP:-1}"     # attention data-parallel lanes (ATTN_TP=4: one tensor-parallel lane)
fastafd_run_bench
