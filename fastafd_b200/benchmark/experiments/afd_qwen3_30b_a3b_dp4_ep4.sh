#!/usr/bin/env bash
# Qwen3-30B-A3B bf16, 4 attention GPUs as data-parallel lanes + 4 expert GPUs, 64 requests per attention GPU, 1K context.
source "$(dirname "${BASH_SOURCE[0]}")/common.sh"
export PRESET_NAME="afd_qwen3_30b_a3b_dp4_ep4"
export MODEL="${MODEL:-qwen3-30b-a3b}"
export PROMPT_LEN="${PROMPT_LEN:-1024}"
export PER_ATTN_GPU_BSZ="${PER_ATTN_GPU_BSZ:-64}"
export NUM_GPUS="${NUM_GPUS:-8}"
export ATTN_GPUS="${ATTN_GPUS:-4}"
export ATTN_TP="${ATTN_TP:-1}"
export SUITE_NAME="${SUITE_NAME:-qwen3-30b-bf16-1k-1to1}"
fastafd_run_bench
