#!/usr/bin/env bash
# Qwen3-235B-A22B-FP8 with an EAGLE-3 draft head: verify steps of 4 tokens, acceptance fixed at 1.8 for timing.
source "$(dirname "${BASH_SOURCE[0]}")/common.sh"
export PRESET_NAME="afd_qwen3_235b_a22b_fp8_8k_spec4"
export MODEL="${MODEL:-qwen3-235b-a22b-fp8}"
export PROMPT_LEN="${PROMPT_LEN:-8192}"
export PER_ATTN_GPU_BSZ="${PER_ATTN_GPU_BSZ:-88}"
export NUM_GPUS="${NUM_GPUS:-8}"
export ATTN_GPUS="${ATTN_GPUS:-4}"
export NUM_MB="${NUM_MB:-2}"
export STEPS="${STEPS:-32}"
export SPEC_BLOCK="${SPEC_BLOCK:-4}"
export SPEC_ACCEPT="${SPEC_ACCEPT:-1.8}"
export ATTN_TP="${ATTN_TP:-1}"     # attention data-parallel lanes (ATTN_TP=4: one tensor-parallel lane)
fastafd_run_bench
