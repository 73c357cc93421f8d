#!/usr/bin/env bash
# The four arms of the paired validation (optimised path and library path, seeds 1 and 2), each followed by its
# held-out evaluation, then the summary and the verdict.
# Prerequisite: $VAL_DIR/heldout/heldout.pt (python -m faster_yoco_b200.validation.heldout ...).
# environment: DATA_DIR, VAL_DIR; optional ARMS (default: opt ref ref_s2 opt_s2), NPROC, PYTHON
set -u
: "${DATA_DIR:?Set DATA_DIR}" "${VAL_DIR:?Set VAL_DIR}"
HERE=$(cd -- "$(dirname -- "${BASH_SOURCE[0]}")" && pwd)
REPO=$(cd "$HERE/../.." && pwd)
PY=${PYTHON:-python}
for ARM in ${ARMS:-opt ref ref_s2 opt_s2}; do
    case $ARM in
        opt)    bash "$HERE/run_arm.sh" opt    1 b200_fused ;;
        opt_s2) bash "$HERE/run_arm.sh" opt_s2 2 b200_fused ;;
        ref)    bash "$HERE/run_arm.sh" ref    1 torch_baseline ;;
        ref_s2) bash "$HERE/run_arm.sh" ref_s2 2 torch_baseline ;;
        *) echo "unknown arm $ARM" >&2; exit 2 ;;
    esac
    echo "$(date '+%F %T') $ARM training rc=$?"
    (cd "$REPO" && "$PY" -m torch.distributed.run --nnodes=1 --nproc-per-node="${NPROC:-8}" --master-addr 127.0.0.1 \
        --master-port $((20000 + RANDOM % 20000)) -m faster_yoco_b200.validation.eval_ckpt \
        "$VAL_DIR/heldout/heldout.pt" "$VAL_DIR/$ARM/eval.json" $(ls "$VAL_DIR/$ARM"/ckpt/model_*.pt | sort) \
        > "$VAL_DIR/$ARM/eval.log" 2>&1)
    echo "$(date '+%F %T') $ARM evaluation rc=$?"
done
(cd "$REPO" && "$PY" -m faster_yoco_b200.validation.analyze "$VAL_DIR" && "$PY" -m faster_yoco_b200.validation.verdict "$VAL_DIR")
