#!/usr/bin/env bash
# MiniMax-M2.5-FP8 decode replay, 16K context, 36 requests per attention GPU.
source "$(dirname "${BASH_SOURCE[0]}")/common.sh"
export PRESET_NAME="afd_minimax_m25_fp8_16k_b36"
export MODEL="${MODEL:-minimax-m2.5-fp8}"
export PROMPT_LEN="${PROMPT_LEN:-16384}"
export PER_ATTN_GPU_BSZ="${PER_ATTN_GPU_BSZ:-36}"
export NUM_GPUS="${NUM_GPUS:-8}"
export ATTN_GPUS="${ATTN_GPUS:-4}"
export NUM_MB="${NUM_MB:-2}"
export STEPS="${STEPS:-32}"
export ATTN_TP="${ATTN_TP:-1}"     # attention data-parallel lanes (ATTN_TP=4: one tensor-parallel lane)
fastafd_run_bench
