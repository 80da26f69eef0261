#!/usr/bin/env bash
# Qwen3-30B-A3B bf16 on one GPU (attention and experts together): the point the reference arm is compared at.
source "$(dirname "${BASH_SOURCE[0]}")/common.sh"
export PRESET_NAME="colocated_qwen3_30b_a3b"
export MODEL="${MODEL:-qwen3-30b-a3b}"
export PROMPT_LEN="${PROMPT_LEN:-1024}"
export PER_ATTN_GPU_BSZ="${PER_ATTN_GPU_BSZ:-64}"
export NUM_GPUS="${NUM_GPUS:-1}"
export SUITE_NAME="${SUITE_NAME:-qwen3-30b-bf16-1k-colocated}"
fastafd_run_bench
