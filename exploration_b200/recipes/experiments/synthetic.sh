#!/usr/bin/env bash
# Synthetic long-context recipes (S1: MQAR, S2: passkey) for the 2.4M-parameter
# Stack model (Lx2,G, d = 256), three seeds each:
#   * MQAR, 16 single-token keys and 16 queries: ignition at length 128, then
#     training at 512 from those weights;
#   * passkey: training at 512;
#   * zero-shot evaluation of both from 512 up to 16M tokens (fp32, paged
#     sparse read; the planner picks the KV tier: GPU, pinned host or disk).
# Chunk recomputation and ZeRO-1 are off: neither pays at this model size.
# Logs and checkpoints go to runs/. Run from anywhere:
#   bash exploration_b200/recipes/experiments/synthetic.sh
# (Counterpart of the reference's scripts/experiments/synthetic.sh.)
set -euo pipefail
cd "$(dirname "${BASH_SOURCE[0]}")/../../.."
mkdir -p runs
note() { printf '\n== [%s] %s ==\n' "$(date '+%F %T')" "$*"; }
st() { python -m exploration_b200 "$@"; }
small=(--no-checkpoint-chunks --no-optimizer-shard --precision bf16 --batch-size 64 --eval-every 500 --eval-batches 4)
lengths=(512 4096 65536 1000000 2000000 4000000 8000000 16000000)

for seed in 0 2 4; do
  note "S1 MQAR seed $seed"
  st train --task mqar --length 128 --npairs 16 --nqueries 16 --steps 3000 --lr 1e-3 --seed "$seed" \
    --save "runs/s1_mqar128_s$seed.pt" --log "runs/s1_mqar128_s$seed.jsonl" "${small[@]}"
  st train --task mqar --length 512 --npairs 16 --nqueries 16 --steps 6000 --lr 5e-4 --seed "$seed" \
    --weights-only --resume "runs/s1_mqar128_s$seed.pt" --save "runs/s1_mqar512_s$seed.pt" \
    --log "runs/s1_mqar512_s$seed.jsonl" "${small[@]}"
  for n in "${lengths[@]}"; do
    st eval --task mqar --length "$n" --npairs 16 --nqueries 16 --resume "runs/s1_mqar512_s$seed.pt" \
      --batch-size 1 --seed "$seed" --precision fp32 --eval-batches 8 --log "runs/s1_mqar512_s$seed.eval.jsonl"
  done

  note "S2 passkey seed $seed"
  st train --task passkey --length 512 --steps 3000 --lr 5e-4 --seed "$seed" \
    --save "runs/s2_passkey512_s$seed.pt" --log "runs/s2_passkey512_s$seed.jsonl" "${small[@]}"
  for n in "${lengths[@]}"; do
    st eval --task passkey --length "$n" --resume "runs/s2_passkey512_s$seed.pt" --batch-size 1 \
      --seed "$seed" --precision fp32 --eval-batches 8 --log "runs/s2_passkey512_s$seed.eval.jsonl"
  done
done
note "synthetic recipes done"
