#!/usr/bin/env bash
# Write-side (L) x read-side (G) scaling matrix on enwik8: Stack d = 256 with
# arch Lx{1,2,4,8},Gx{1,2,4} (independent weights) against a baseline with
# about the same parameter count (layer counts in BASE below, the
# reference's matrix). Length 4096,
# batch 16, 8000 steps, lr 5e-4, bf16, seed 0; eval at 4096 during training
# and zero-shot at 16k and 65k (fp32). Cells are split over WORKERS GPUs.
# Summary: python -m exploration_b200.recipes.experiments.scaling_matrix_report
# (Counterpart of the reference's scripts/experiments/scaling_matrix.sh; this
# one leaves the machine running when it finishes.)
set -euo pipefail
cd "$(dirname "${BASH_SOURCE[0]}")/../../.."
mkdir -p runs
WORKERS=${WORKERS:-2}
note() { printf '\n== [%s] %s ==\n' "$(date '+%F %T')" "$*"; }
common=(--task enwik8 --length 4096 --batch-size 16 --steps 8000 --lr 5e-4 --precision bf16
        --no-checkpoint-chunks --no-optimizer-shard --eval-every 500 --eval-batches 4)

declare -A BASE=([l1g1]=2 [l2g1]=3 [l4g1]=5 [l8g1]=9 [l1g2]=3 [l2g2]=4 [l4g2]=6 [l8g2]=10
                 [l1g4]=5 [l2g4]=6 [l4g4]=8 [l8g4]=13)

cell() {   # cell <L> <G> <gpu>
  local l=$1 g=$2 gpu=$3 name="l${1}g${2}"
  local arch layers=${BASE[$name]}
  arch=$([ "$l" = 1 ] && echo L || echo "Lx$l"),$([ "$g" = 1 ] && echo G || echo "Gx$g")
  note "cell $name arch=$arch baseline_layers=$layers gpu=$gpu"
  CUDA_VISIBLE_DEVICES=$gpu python -m exploration_b200 train --arch "$arch" "${common[@]}" \
    --save "runs/sc_$name.pt" --log "runs/sc_$name.jsonl"
  CUDA_VISIBLE_DEVICES=$gpu python -m exploration_b200 train --model baseline --layers "$layers" "${common[@]}" \
    --save "runs/sc_${name}_base.pt" --log "runs/sc_${name}_base.jsonl"
  for n in 16384 65536; do
    CUDA_VISIBLE_DEVICES=$gpu python -m exploration_b200 eval --task enwik8 --length "$n" \
      --resume "runs/sc_$name.pt" --batch-size 2 --precision fp32 --eval-batches 4 --log "runs/sc_$name.jsonl"
    CUDA_VISIBLE_DEVICES=$gpu python -m exploration_b200 eval --model baseline --task enwik8 --length "$n" \
      --resume "runs/sc_${name}_base.pt" --batch-size 2 --precision fp32 --eval-batches 4 \
      --log "runs/sc_${name}_base.jsonl"
  done
}

i=0
for g in 1 2 4; do
  for l in 1 2 4 8; do
    cell "$l" "$g" $(( i % WORKERS )) &
    i=$(( i + 1 ))
    if (( i % WORKERS == 0 )); then wait; fi
  done
done
wait
note "scaling matrix done"
