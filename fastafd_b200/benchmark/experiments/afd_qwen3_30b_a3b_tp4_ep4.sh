#!/usr/bin/env bash
# Qwen3-30B-A3B bf16, one attention lane tensor-parallel over 4 GPUs + 4 expert GPUs (fused collectives).
source "$(dirname "${BASH_SOURCE[0]}")/common.sh"
export PRESET_NAME="afd_qwen3_30b_a3b_tp4_ep4"
export MODEL="${MODEL:-qwen3-30b-a3b}"
export PROMPT_LEN="${PROMPT_LEN:-1024}"
export PER_ATTN_GPU_BSZ="${PER_ATTN_GPU_BSZ:-64}"
export NUM_GPUS="${NUM_GPUS:-8}"
export ATTN_GPUS="${ATTN_GPUS:-4}"
export ATTN_TP="${ATTN_TP:-4}"
export TP_FUSED="${TP_FUSED:-1}"
export SUITE_NAME="${SUITE_NAME:-qwen3-30b-bf16-1k-tp4}"
fastafd_run_bench
