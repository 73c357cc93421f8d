#!/usr/bin/env bash
# YOCO-3B pretraining with the reference recipe's arguments on one node of B200s.
# usage: DATA_DIR=/path/to/Data OUTPUT_DIR=/path/to/out [NPROC=8] [PRESET=b200_fused] \
#        bash faster_yoco_b200/cli/train_yoco_3b.sh [extra train arguments, e.g. --max-update 20000]
set -euo pipefail
: "${DATA_DIR:?Set DATA_DIR to the training data root that contains json/train.json}"
: "${OUTPUT_DIR:?Set OUTPUT_DIR to the output directory}"
NPROC=${NPROC:-8}
[[ -f "$DATA_DIR/json/train.json" ]] || { echo "Missing $DATA_DIR/json/train.json" >&2; exit 2; }
mkdir -p "$OUTPUT_DIR"
REPO=$(cd -- "$(dirname -- "${BASH_SOURCE[0]}")/../.." && pwd)
cd "$REPO"
python -m torch.distributed.run --nnodes=1 --nproc-per-node="$NPROC" --master-addr 127.0.0.1 \
    --master-port "${MASTER_PORT:-29501}" -m faster_yoco_b200.cli.train "$DATA_DIR" \
    --preset "${PRESET:-b200_fused}" \
    --save-interval-updates 5000 --no-epoch-checkpoints --arch yoco_3b --criterion cross_entropy --task gpt \
    --tokens-per-sample 2048 --tokenizer-pad-to-multiple 8 --pad-to-max-len \
    --optimizer adam --adam-betas "(0.9, 0.95)" --adam-eps 1e-06 --clip-norm 2.0 --lr 0.00015 \
    --lr-scheduler polynomial_decay --warmup-updates 50 --weight-decay 0.05 --batch-size 1 \
    --model-parallel-size 1 --update-freq 1 --batch-read-ahead 1000 --total-num-update 300000 \
    --log-format simple --log-interval 10 --disable-validation --tiktoken-model cl100k_base --no-save --bf16 \
    --zero-sharding os --seed 1 --save-dir "$OUTPUT_DIR/checkpoints" \
    "$@" 2>&1 | tee -a "$OUTPUT_DIR/train.log"
exit "${PIPESTATUS[0]}"
