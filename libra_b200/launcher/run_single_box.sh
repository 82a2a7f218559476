#!/usr/bin/env bash
# Launch an async GRPO run on one 8x B200 box.
#   bash libra_b200/launcher/run_single_box.sh <config.yaml> [extra trainer args]
# Rollout servers (HTTP backend) start on the rollout GPUs first; the trainer
# runs under torch.distributed.run on the training GPUs.
set -euo pipefail
CONFIG=${1:?usage: run_single_box.sh <config.yaml>}
shift || true
export NCCL_DEBUG=${NCCL_DEBUG:-WARN}
export TORCH_NCCL_ASYNC_ERROR_HANDLING=${TORCH_NCCL_ASYNC_ERROR_HANDLING:-1}
exec python -m libra_b200.launcher.box_launcher --config "$CONFIG" "$@"
