#!/bin/bash
# Launch one of the benchmarks on every GPU of this node (reference: scripts/run_benchmark.sh,
# which prepares the environment for the inter-node benchmarks).
#   examples/run_benchmark.sh benchmarks/expert_transfer.py --balance uneven_intranode
#   NGPU=2 examples/run_benchmark.sh benchmarks/bench_speculative.py --layers 4
# One process per GPU; a short NCCL timeout plus an outer `timeout` end a run whose ranks
# wait on a lost peer.
set -euo pipefail
cd "$(dirname "$0")/.."
BENCH="${1:?usage: examples/run_benchmark.sh <benchmark.py> [args...]}"
shift
export LOGS="${LOGS:-logs/$(date +%Y-%m-%d_%H-%M-%S)}"
mkdir -p "$LOGS"
NGPU="${NGPU:-$(nvidia-smi -L | wc -l)}"
timeout -k 60 "${TIMEOUT:-1800}" python -m torch.distributed.run --nnodes=1 --nproc-per-node "$NGPU" \
    --master-addr 127.0.0.1 --master-port "${MASTER_PORT:-29501}" \
    "$BENCH" "$@" 2>&1 | tee "$LOGS/$(basename "$BENCH" .py).log"
