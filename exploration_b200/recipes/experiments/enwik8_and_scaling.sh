#!/usr/bin/env bash
# enwik8 recipes ("train dense, infer sparse"; top-k only matters at eval):
#   E1  Stack vs baseline dense LM at 512, zero-shot to 4k/16k/65k; baseline
#       passkey and MQAR references
#   E2  L-layer and G-round scans (shared-weight cycles and independent rounds)
#   E3  block size 8..64
#   E4  harder MQAR (pair count grows with length, two-token keys)
#   E5  training length 256..2048 at block 32
# Needs data/enwik8 (see exploration_b200.data.tokens). Checkpoints in runs/.
# (Counterpart of the reference's scripts/experiments/enwik8_and_scaling.sh.)
set -euo pipefail
cd "$(dirname "${BASH_SOURCE[0]}")/../../.."
mkdir -p runs
note() { printf '\n== [%s] %s ==\n' "$(date '+%F %T')" "$*"; }
st() { python -m exploration_b200 "$@"; }
lm=(--task enwik8 --length 512 --batch-size 32 --lr 5e-4 --precision bf16 --eval-every 500 --eval-batches 4)
zero_shot() {   # zero_shot <checkpoint> <task> <lengths...> (extra eval flags in EVAL_FLAGS)
  local ck=$1 task=$2; shift 2
  for n in "$@"; do
    st eval --task "$task" --length "$n" --resume "$ck" --batch-size 2 --precision fp32 --eval-batches 8 ${EVAL_FLAGS:-}
  done
}
tag() { echo "${1//[^A-Za-z0-9]/_}"; }

note "E1 dense LM at 512"
st train --model stack --arch Lx2,G --steps 30000 --save runs/e1_stack.pt "${lm[@]}"
st train --model baseline --layers 3 --steps 30000 --save runs/e1_base.pt "${lm[@]}"
zero_shot runs/e1_stack.pt enwik8 4096 16384 65536
for n in 4096 16384 65536; do
  st eval --model baseline --task enwik8 --length "$n" --resume runs/e1_base.pt --batch-size 2 --precision fp32 --eval-batches 8
done
st train --model baseline --task passkey --length 512 --steps 1500 --batch-size 64 --lr 5e-4 --precision bf16 \
  --eval-every 500 --eval-batches 4 --save runs/e1_base_passkey.pt
st train --model baseline --task mqar --length 128 --npairs 16 --nqueries 16 --steps 3000 --batch-size 64 --lr 1e-3 \
  --precision bf16 --eval-every 500 --eval-batches 4 --save runs/e1_base_mqar.pt

note "E2 L and G scans"
for arch in "L,G" "Lx2,G" "Lx4,G" "Lx8,G" "(L)x4,G" "Lx2,(G)x2" "Lx2,(G)x4" "Lx2,(G)x8" "Lx2,Gx4"; do
  ck="runs/e2_$(tag "$arch").pt"
  st train --model stack --arch "$arch" --steps 8000 --save "$ck" "${lm[@]}"
  zero_shot "$ck" enwik8 4096 65536
done

note "E3 block size"
for b in 8 16 32 64; do
  st train --model stack --arch Lx2,G --block-size "$b" --topk 64 --steps 8000 --save "runs/e3_b$b.pt" "${lm[@]}"
  zero_shot "runs/e3_b$b.pt" enwik8 4096 65536
done

note "E4 harder MQAR"
hard=(--npairs-density 0.03125 --nkeytoks 2 --nqueries 16)
st train --model stack --task mqar --length 512 "${hard[@]}" --steps 3000 --batch-size 64 --lr 1e-3 --precision bf16 \
  --eval-every 500 --eval-batches 4 --stop-exact 0.99 --save runs/e4_stack.pt
st train --model baseline --layers 3 --task mqar --length 512 "${hard[@]}" --steps 3000 --batch-size 64 --lr 1e-3 \
  --precision bf16 --eval-every 500 --eval-batches 4 --save runs/e4_base.pt
EVAL_FLAGS="${hard[*]}" zero_shot runs/e4_stack.pt mqar 4096 16384 65536
for n in 4096 16384 65536; do
  st eval --model baseline --task mqar --length "$n" "${hard[@]}" --resume runs/e4_base.pt --batch-size 2 \
    --precision fp32 --eval-batches 8
done

note "E5 training length at block 32"
for n in 256 512 1024 2048; do
  st train --model stack --task enwik8 --length "$n" --block-size 32 --topk 64 --arch Lx2,G --batch-size 32 \
    --steps 8000 --lr 5e-4 --precision bf16 --eval-every 500 --eval-batches 4 --save "runs/e5_n$n.pt"
  zero_shot "runs/e5_n$n.pt" enwik8 4096 16384 65536
done
note "enwik8 recipes done"
