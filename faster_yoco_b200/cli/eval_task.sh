#!/usr/bin/env bash
# Multiple-choice evaluation of a checkpoint on one harness task.
# usage: TASK=harness_boolq DATA=harness_data/ CKPT_DIR=/path/YOCO-3B-1M bash faster_yoco_b200/cli/eval_task.sh
set -euo pipefail
REPO=$(cd -- "$(dirname -- "${BASH_SOURCE[0]}")/../.." && pwd)
cd "$REPO"
python -m torch.distributed.run --nnodes=1 --nproc-per-node="${NPROC:-1}" --master-addr 127.0.0.1 \
    --master-port "${MASTER_PORT:-29505}" -m faster_yoco_b200.cli.validate \
    --data-dir "${DATA:?Set DATA to the harness data directory}" --criterion harness_eval --task harness_eval \
    --batch-size 4 --eval-data "${TASK:-harness_boolq}" --log-format simple --log-interval 10 --bf16 \
    --tokenizer-pad-to-multiple 8 --arch yoco_3b --tiktoken-model cl100k_base \
    --load-ckpt "${CKPT_DIR:?Set CKPT_DIR}/checkpoint.pth" --yoco-model "$CKPT_DIR" --tokens-per-sample 4096 "$@"
