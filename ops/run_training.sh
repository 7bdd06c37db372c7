#!/usr/bin/env bash
# Launch (or resume) the production defense-training service on one or more GPUs.
#
#   ops/run_training.sh DEVICE_OR_GPUS SEED OUTPUT_DIR
#
# DEVICE_OR_GPUS is a device string ("cuda:0") for one process, or a GPU count
# ("8") for one process per GPU under torchrun. A run directory that already
# holds policy.pt resumes from it (--initial-checkpoint). Environment:
#   PYTHON            interpreter (default: python3 on PATH)
#   AUTODRIVE_ROOT    repository root (default: this script's parent directory)
#   MASTER_PORT       rendezvous port for multi-GPU runs (default 29531)
set -euo pipefail

if [[ $# -ne 3 ]]; then
    echo "usage: $0 DEVICE_OR_GPUS SEED OUTPUT_DIR" >&2
    exit 2
fi
target=$1
seed=$2
output=$3
root=${AUTODRIVE_ROOT:-$(cd "$(dirname "$0")/.." && pwd)}
python_bin=${PYTHON:-python3}
checkpoint="$output/policy.pt"
cd "$root"

train_args=(train --task defense --algorithm generational --architecture strategic_adstar
    --generations 40 --opponent-pool-size 8 --strong-checkpoints 2 --envs 24 --horizon 8000
    --seed "$seed" --output "$output")
if [[ -s "$checkpoint" ]]; then
    train_args+=(--initial-checkpoint "$checkpoint")
fi

if [[ "$target" =~ ^[0-9]+$ ]]; then
    exec "$python_bin" -m torch.distributed.run --nnodes=1 --nproc-per-node "$target" \
        --master-addr 127.0.0.1 --master-port "${MASTER_PORT:-29531}" \
        -m autodrive_b200.train.cli "${train_args[@]}" --device cuda
fi
exec "$python_bin" -m autodrive_b200.train.cli "${train_args[@]}" --device "$target"
