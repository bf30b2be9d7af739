#!/bin/bash
# HF Qwen3-MoE smoke run with the fused expert-parallel blocks swapped in
# (reference: scripts/run_hf.sh). Single process, one GPU.
set -euo pipefail
cd "$(dirname "$0")/.."
timeout -k 30 "${TIMEOUT:-900}" python examples/hf_qwen.py "$@"
