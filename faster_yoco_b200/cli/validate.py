"""Evaluation entry point (yoco/validate.py:44-293): builds task / model / criterion, casts to bf16, runs the
criterion over the task's batches and prints the reduced metrics. ``--profile`` wraps the run in NVTX ranges.

    python -m faster_yoco_b200.cli.validate --task harness_eval --criterion harness_eval --eval-data harness_boolq \\
        --data-dir harness_data/ --batch-size 4 --bf16 --arch yoco_3b --tiktoken-model cl100k_base \\
        --yoco-model CKPT_DIR --load-ckpt CKPT_DIR/checkpoint.pth --tokens-per-sample 4096
    python -m faster_yoco_b200.cli.validate --task pseudo --criterion multi_needle --needle-num 4 ...
"""
from __future__ import annotations

import json
import sys

import torch
import torch.distributed as dist

from ..parallel import dist as D
from ..registry import get_criterion
from ..utils.tracing import emit_nvtx
from .common import build_model, build_task, setup_runtime
from .options import validate_parser


def build_criterion(args, task, family):
    cls = get_criterion(args.criterion)
    if args.criterion in ("needle_haystack", "multi_needle"):
        kw = dict(tokens_per_sample=args.tokens_per_sample, interval=args.interval,
                  needle_file_path=args.needle_file_path or "", yoco=family == "yoco")
        if args.criterion == "multi_needle":
            kw["needle_num"] = args.needle_num
        return cls(task, **kw)
    return cls(task)


def _to_device(sample, device):
    if isinstance(sample, dict):
        return {k: _to_device(v, device) for k, v in sample.items()}
    if torch.is_tensor(sample):
        return sample.to(device, non_blocking=True)
    return sample


def main(argv=None) -> int:
    args = validate_parser().parse_args(argv)
    device = setup_runtime(args)
    rank, world = D.rank(), D.world()
    tp = max(1, int(getattr(args, "model_parallel_size", 1) or 1))
    task = build_task(args)
    model, family = build_model(args, task, device)
    model.eval()
    crit = build_criterion(args, task, family)
    results = {}
    with emit_nvtx(args.profile):
        if args.criterion in ("needle_haystack", "multi_needle"):
            _, _, log = crit(model, None, device=device)
            logs = [log]
        else:
            ds = task.load_dataset(args.valid_subset)
            # the ranks of one tensor-parallel group evaluate the same batches (consecutive ranks form a group)
            itr = task.get_batch_iterator(ds, max_sentences=args.batch_size, seed=args.seed, num_shards=world // tp,
                                          shard_id=rank // tp)
            logs = []
            for i, sample in enumerate(itr):
                if args.max_valid_steps is not None and i >= args.max_valid_steps:
                    break
                with torch.no_grad():
                    _, _, log = crit(model, _to_device(sample, device))
                logs.append({k: (float(v) if torch.is_tensor(v) else v) for k, v in log.items()})
            if hasattr(itr, "close"):
                itr.close()
    if D.is_dist():
        gathered = [None] * world
        dist.all_gather_object(gathered, logs)
        logs = [l for g, part in enumerate(gathered) if g % tp == 0 for l in part]   # one copy per replica
    results = type(crit).reduce_metrics(logs)
    if rank == 0:
        print(json.dumps({"subset": args.valid_subset, "task": args.task, "criterion": args.criterion,
                          **results}, default=str), flush=True)
    D.barrier()
    D.destroy()
    return 0


def cli_main():
    sys.exit(main())


if __name__ == "__main__":
    cli_main()
