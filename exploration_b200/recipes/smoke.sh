#!/usr/bin/env bash
# End-to-end smoke run on small inputs (after validate.sh):
#   GPUS=2 bash exploration_b200/recipes/smoke.sh
# Four optimizer steps with gradient accumulation and periodic saves, a
# reload into paged sparse evaluation, then the operator benchmarks
# (dense through the eager oracle and the native kernels, sparse at 65,536
# keys). (Counterpart of the reference's scripts/remote_smoke.sh.)
set -euo pipefail
cd "$(dirname "${BASH_SOURCE[0]}")/../.."
GPUS=${GPUS:-1}
REPORT_DIR=${REPORT_DIR:-runs/smoke}
mkdir -p "$REPORT_DIR"

torchrun --standalone --local-addr 127.0.0.1 --nproc_per_node="$GPUS" -m exploration_b200 train \
  --config configs/stack_2m.json --task random --length 512 --steps 4 --grad-accum 2 \
  --save-every 2 --save "$REPORT_DIR/model.pt" --log-every 1 2>&1 | tee "$REPORT_DIR/train.log"

python -m exploration_b200 eval --resume "$REPORT_DIR/model.pt" --task random --length 2048 \
  --eval-positions 16 --cache cpu --output "$REPORT_DIR/eval.json" 2>&1 | tee "$REPORT_DIR/eval.log"

for spec in "dense eager 512 eager" "dense cuda 512 native" "sparse cuda 65536 sparse"; do
  set -- $spec
  python -m exploration_b200 benchmark --operation "$1" --backend "$2" --length "$3" \
    --output "$REPORT_DIR/$4.json"
done
