#!/usr/bin/env bash
# Training profiles (train_best.sh of the reference), expressed as overrides
# of the full_g4 preset.  Extra arguments are passed to `main.py train`.
# Multi-GPU: set NPROC (default: number of visible GPUs) to launch with torchrun.
set -euo pipefail
cd "$(dirname "$0")"

NPROC="${NPROC:-$(python -c 'import torch; print(max(1, torch.cuda.device_count()))')}"
run() {
  if [ "$NPROC" -gt 1 ]; then
    python -m torch.distributed.run --nnodes=1 --nproc-per-node "$NPROC" \
      --master-addr 127.0.0.1 --master-port "${MASTER_PORT:-29500}" main.py train "$@"
  else
    python main.py train "$@"
  fi
}

# quality: top-4, shared expert 2x routed width, batch 8
quality()       { run --config full_g4 --n_active 4 --d_ff 1536 --d_ff_dense 3072 --batch 8 "$@"; }
# quality + throughput: top-2, 10 dense layers, batch 16
quality_speed() { run --config full_g4 --n_active 2 --d_ff 1536 --d_ff_dense 2048 --dense_layers 10 --batch 16 "$@"; }
# balanced: top-1, small routed experts, wide shared expert
balanced()      { run --config full_g4 --n_active 1 --d_ff 768 --d_ff_dense 4096 --dense_layers 10 --batch 16 "$@"; }
# throughput: top-1, 14 dense layers
throughput()    { run --config full_g4 --n_active 1 --d_ff 1536 --d_ff_dense 2048 --dense_layers 14 --batch 16 "$@"; }
# MFU benchmark only: a very wide shared expert
mfu()           { run --config full_g4 --n_active 1 --d_ff 1536 --d_ff_dense 16384 --dense_layers 10 --batch 8 "$@"; }

usage() {
  cat <<EOF
Usage: $0 <profile> [extra args for main.py train]
Profiles: quality | quality_speed | balanced | throughput | mfu
EOF
}

case "${1:-}" in
  quality)       shift; quality "$@" ;;
  quality_speed) shift; quality_speed "$@" ;;
  balanced)      shift; balanced "$@" ;;
  throughput)    shift; throughput "$@" ;;
  mfu)           shift; mfu "$@" ;;
  -h|--help)     usage ;;
  *)             usage; exit 1 ;;
esac
