#!/usr/bin/env bash
# Throughput of the Stack model against the same-size SDPA baseline, plus the
# dense operator comparison (eager oracle / torch / native):
#   GPUS=2 LENGTH=8192 STEPS=24 bash exploration_b200/recipes/camera_ready.sh
# CHECKPOINT=1 turns on chunk recomputation for both models. JSONL logs (one
# record per step with tokens_per_second and peak memory) go to REPORT_DIR.
# (Counterpart of the reference's scripts/benchmark_camera_ready.sh.)
set -euo pipefail
cd "$(dirname "${BASH_SOURCE[0]}")/../.."
GPUS=${GPUS:-2}
LENGTH=${LENGTH:-8192}
STEPS=${STEPS:-24}
LOG_EVERY=${LOG_EVERY:-8}
REPORT_DIR=${REPORT_DIR:-runs/benchmarks/camera-ready}
mkdir -p "$REPORT_DIR"
if [[ "${CHECKPOINT:-0}" == 1 ]]; then recompute=--checkpoint-chunks; else recompute=--no-checkpoint-chunks; fi
shared=(--task random --length "$LENGTH" --batch-size 1 --steps "$STEPS" --grad-accum 1
        --log-every "$LOG_EVERY" --save '' --precision bf16 "$recompute" --backend auto)
launch=(torchrun --standalone --local-addr 127.0.0.1 --nproc_per_node="$GPUS" -m exploration_b200 train)

"${launch[@]}" --model stack --config configs/stack_2m.json "${shared[@]}" > "$REPORT_DIR/stack.jsonl" 2>&1
"${launch[@]}" --model baseline --config configs/baseline_2m.json --flash-attention auto "${shared[@]}" \
  > "$REPORT_DIR/baseline.jsonl" 2>&1
python -m exploration_b200 benchmark --compare --operation dense --length 512 \
  --output "$REPORT_DIR/dense-operator.json"
echo "reports in $REPORT_DIR"
