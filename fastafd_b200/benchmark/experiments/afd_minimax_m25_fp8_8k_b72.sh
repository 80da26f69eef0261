#!/usr/bin/env bash
# MiniMax-M2.5-FP8 decode replay, 8K context, 72 requests per attention GPU; second pass with Zipf-skewed routing.
source "$(dirname "${BASH_SOURCE[0]}")/common.sh"
export PRESET_NAME="afd_minimax_m25_fp8_8k_b72"
export MODEL="${MODEL:-minimax-m2.5-fp8}"
export PROMPT_LEN="${PROMPT_LEN:-8192}"
export PER_ATTN_GPU_BSZ="${PER_ATTN_GPU_BSZ:-72}"
export NUM_GPUS="${NUM_GPUS:-8}"
export ATTN_GPUS="${ATTN_GPUS:-4}"
export NUM_MB="${NUM_MB:-2}"
export STEPS="${STEPS:-32}"
export ROUTER_BIAS="${ROUTER_BIAS:-zipf:1.2}"
export ATTN_TP="${ATTN_TP:-1}"     # attention data-parallel lanes (ATTN_TP=4: one tensor-parallel lane)
fastafd_run_bench
