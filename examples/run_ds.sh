#!/bin/bash
# Launch the MoE driver on every GPU of one node (reference: scripts/run_ds.sh).
# One process per GPU; NCCL for bootstrap and dense gradients, NVLink peer stores for EP.
set -euo pipefail
cd "$(dirname "$0")/.."
export LOGS="${LOGS:-logs/$(date +%Y-%m-%d_%H-%M-%S)}"
mkdir -p "$LOGS/profile"
NGPU="${NGPU:-$(nvidia-smi -L | wc -l)}"
CONFIG="${CONFIG:-configs/qwen3_30b_a3b_ep8_sepx.json}"
timeout -k 60 "${TIMEOUT:-3600}" python -m torch.distributed.run --nnodes=1 --nproc-per-node "$NGPU" \
    --master-addr 127.0.0.1 --master-port "${MASTER_PORT:-29500}" \
    examples/ds_moe.py --config-pth "$CONFIG" "$@" 2>&1 | tee "$LOGS/run.log"
