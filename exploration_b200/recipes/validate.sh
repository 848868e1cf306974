#!/usr/bin/env bash
# Correctness checks on a CUDA host, from the repository root:
#   GPUS=8 bash exploration_b200/recipes/validate.sh
# CPU reference suite, the sm_100a resource and parity suites, then the
# distributed gradient-parity suite at every context-parallel size the GPU
# count allows (CP=2, CP=2 x DP=2, CP=4, CP=8). Reports go to REPORT_DIR.
# Nothing is installed, downloaded or shut down.
# (Counterpart of the reference's scripts/remote_validate.sh.)
set -euo pipefail
cd "$(dirname "${BASH_SOURCE[0]}")/../.."
GPUS=${GPUS:-1}
REPORT_DIR=${REPORT_DIR:-runs/validation}
mkdir -p "$REPORT_DIR"

run() {   # run <name> <command...>: JSON report + log per suite
  local name=$1; shift
  "$@" --output "$REPORT_DIR/$name.json" 2>&1 | tee "$REPORT_DIR/$name.log"
}
distributed() {   # distributed <ranks> <cp> <name>
  run "$3" torchrun --standalone --local-addr 127.0.0.1 --nproc_per_node="$1" \
    -m exploration_b200 validate --suite distributed --cp "$2"
}

run reference python -m exploration_b200 validate --suite reference
run resources python -m exploration_b200 validate --suite resources
run cuda python -m exploration_b200 validate --suite cuda
if [ "$GPUS" -ge 2 ]; then distributed 2 2 distributed_cp2; fi
if [ "$GPUS" -ge 4 ]; then
  distributed 4 2 distributed_cp2_dp2
  distributed 4 4 distributed_cp4
fi
if [ "$GPUS" -ge 8 ]; then distributed 8 8 distributed_cp8; fi
