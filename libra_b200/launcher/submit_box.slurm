#!/usr/bin/env bash
#SBATCH --job-name=libra-b200
#SBATCH --nodes=1
#SBATCH --gres=gpu:8
#SBATCH --exclusive
#SBATCH --time=24:00:00
# Slurm wrapper for one 8x B200 node:  sbatch libra_b200/launcher/submit_box.slurm <config.yaml>
set -euo pipefail
CONFIG=${1:?usage: sbatch submit_box.slurm <config.yaml>}
cd "${SLURM_SUBMIT_DIR:-$PWD}"
python -m libra_b200.infra.preflight nccl --gpus 8 || { echo "NCCL preflight failed"; exit 1; }
bash libra_b200/launcher/run_single_box.sh "$CONFIG"
