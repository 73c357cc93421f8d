#!/usr/bin/env bash
# One arm of the paired training validation: the measured YOCO-3B recipe for MAXU updates with bf16 model-only
# checkpoints every SAVEINT updates.
# usage: run_arm.sh <arm name> <seed> <preset: b200_fused | b200_nccl | torch_baseline | ...>
# environment: DATA_DIR (training data root: json/train.json, shard/<source>/*.jsonl), VAL_DIR (output root);
#   optional MAXU (20000), SAVEINT (2000), NPROC (8), MASTER_PORT (random), PYTHON (python)
set -u
ARM=$1; SEED=$2; PRESET=$3
: "${DATA_DIR:?Set DATA_DIR}" "${VAL_DIR:?Set VAL_DIR}"
HERE=$(cd -- "$(dirname -- "${BASH_SOURCE[0]}")" && pwd)
REPO=$(cd "$HERE/../.." && pwd)
PY=${PYTHON:-python}
OUT=$VAL_DIR/$ARM; mkdir -p "$OUT/ckpt"
echo "$(date '+%F %T') start $ARM seed=$SEED preset=$PRESET" >> "$OUT/run.log"
git -C "$REPO" log --oneline -1 >> "$OUT/run.log" 2>/dev/null
T0=$(date +%s)
cd "$REPO"
"$PY" -m torch.distributed.run --nnodes=1 --nproc-per-node="${NPROC:-8}" --master-addr 127.0.0.1 \
    --master-port "${MASTER_PORT:-$((20000 + RANDOM % 20000))}" -m faster_yoco_b200.cli.train "$DATA_DIR" \
    --preset "$PRESET" --arch yoco_3b --criterion cross_entropy --task gpt --tokens-per-sample 2048 \
    --tokenizer-pad-to-multiple 8 --pad-to-max-len --adam-betas '(0.9, 0.95)' --adam-eps 1e-06 --clip-norm 2.0 \
    --lr 0.00015 --warmup-updates 50 --weight-decay 0.05 --batch-size 1 --update-freq 1 --batch-read-ahead 1000 \
    --total-num-update 300000 --log-interval 10 --tiktoken-model cl100k_base --bf16 --seed "$SEED" \
    --save-dir "$OUT/ckpt" --save-model-only --save-interval-updates "${SAVEINT:-2000}" \
    --max-update "${MAXU:-20000}" > "$OUT/train.log" 2>&1
RC=$?
echo "$(date '+%F %T') end $ARM rc=$RC wall_s=$(( $(date +%s) - T0 ))" >> "$OUT/run.log"
exit $RC
