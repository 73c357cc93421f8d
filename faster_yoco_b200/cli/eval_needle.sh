#!/usr/bin/env bash
# Multi-needle retrieval up to 1M tokens (chunked prefill + greedy decoding).
# usage: CKPT_DIR=/path/YOCO-3B-1M ESSAYS=/path/PaulGrahamEssays bash faster_yoco_b200/cli/eval_needle.sh
set -euo pipefail
REPO=$(cd -- "$(dirname -- "${BASH_SOURCE[0]}")/../.." && pwd)
cd "$REPO"
python -m torch.distributed.run --nnodes=1 --nproc-per-node=1 --master-addr 127.0.0.1 \
    --master-port "${MASTER_PORT:-29504}" -m faster_yoco_b200.cli.validate \
    --task pseudo --criterion multi_needle --needle-num "${NEEDLES:-4}" --batch-size 1 --max-epoch 1 --no-save \
    --tiktoken-model cl100k_base --bf16 --arch yoco_3b --load-ckpt "${CKPT_DIR:?Set CKPT_DIR}/checkpoint.pth" \
    --yoco-model "$CKPT_DIR" --needle-file-path "${ESSAYS:?Set ESSAYS}" \
    --tokens-per-sample "${LEN:-1048576}" --interval "${INTERVAL:-1048576}" "$@"
