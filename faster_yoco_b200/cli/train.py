"""Training entry point (the reference's ``yoco/train.py`` -> fairseq ``cli_main``; call stack of one update in
train/trainer.py).

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m faster_yoco_b200.cli.train DATA_DIR --arch yoco_3b \\
        --task gpt --criterion cross_entropy --tokens-per-sample 2048 --batch-size 1 --tiktoken-model cl100k_base \\
        --bf16 --zero-sharding os --max-update 1000

Per update: ``update_freq`` micro-batches from the task's iterator, one ``Trainer.train_step``; a log line every
``--log-interval`` updates (the only host read of device metrics); a checkpoint every ``--save-interval-updates``
(model, consolidated optimizer state, LR schedule, every rank's data-iterator state). A run resumes from
``<save-dir>/<restore-file>`` when it exists.
"""
from __future__ import annotations

import os
import sys
import time
from typing import Optional

import torch
import torch.distributed as dist

from ..config import OptimConfig
from ..parallel import dist as D
from ..parallel.zero import exchange_schedule
from ..train.checkpoint import load_checkpoint, part_path, prune_interval_checkpoints, save_checkpoint
from ..train.metrics import format_log
from ..train.trainer import Trainer
from .common import build_model, build_task, setup_runtime
from .options import parse_with_preset, train_parser


def _cp_slice(batch, cp: int):
    """This rank's contiguous block of every sequence under context parallelism; the token count (the gradient
    normaliser, summed over all ranks) is split so that the blocks of a sequence add up to its count."""
    if cp <= 1:
        return batch
    from ..parallel import context as CP
    r = CP.cp_rank()
    L = batch["src_tokens"].shape[1] // cp
    out = dict(batch)
    out["src_tokens"] = batch["src_tokens"][:, r * L:(r + 1) * L].contiguous()
    out["target"] = batch["target"][:, r * L:(r + 1) * L].contiguous()
    n = int(batch["ntokens"])
    out["ntokens"] = n // cp + (n % cp if r == cp - 1 else 0)
    return out


def _gather_iterator_states(itr):
    st = itr.state_dict() if hasattr(itr, "state_dict") else None
    if not D.is_dist():
        return [st]
    out = [None] * D.world()
    dist.all_gather_object(out, st)
    return out


def _save_model_only(args, model, nu: int, rank: int):
    """bf16 model-only save on data-parallel rank 0 (reference parameter names, ``decoder.model.`` prefix; one part
    file per tensor-parallel rank) and peak memory. ``rank``: this rank's data-parallel rank."""
    import json
    mem = {"rank": rank, "num_updates": nu, "time": time.time()}
    if torch.cuda.is_available():
        mem.update(max_allocated_gib=torch.cuda.max_memory_allocated() / 2 ** 30,
                   max_reserved_gib=torch.cuda.max_memory_reserved() / 2 ** 30)
    print("VALIDATION_MEM " + json.dumps(mem), flush=True)
    path = part_path(os.path.join(args.save_dir, f"model_{nu:06d}.pt"))
    if rank == 0 and nu > 0 and not os.path.exists(path):
        t0 = time.time()
        os.makedirs(args.save_dir, exist_ok=True)
        sd = {"decoder.model." + k: v.detach().to("cpu", copy=True) for k, v in model.state_dict().items()}
        torch.save({"model": sd, "num_updates": nu}, path + ".tmp")
        os.replace(path + ".tmp", path)
        print(f"VALIDATION_CKPT {path} {time.time() - t0:.1f}s", flush=True)


def validate_lm(model, task, args, device, rank: int, world: int, rep: int = 1, cp: int = 1,
                tp: int = 1) -> Optional[dict]:
    """Mean next-token loss (bits) over up to --max-valid-steps batches of the valid subset, summed over ranks
    (fairseq's validation pass of the training loop; no gradients, the module path of the model). The `rep`
    consecutive ranks of one model replica (a context- or tensor-parallel group) read the same batches; under context
    parallelism each takes its block of every sequence."""
    import math
    from .. import ops
    try:
        ds = task.load_dataset(args.valid_subset)
    except (FileNotFoundError, KeyError):
        return None
    if not getattr(ds, "data", None):
        return None                       # an empty source list (the reference corpus layout has one)
    itr = task.get_batch_iterator(ds, max_sentences=args.batch_size, seed=args.seed, num_shards=world // rep,
                                  shard_id=rank // rep, prefetch=0)
    was_training = model.training
    model.eval()
    tot = torch.zeros(2, dtype=torch.float64, device=device)
    with torch.no_grad():
        for _ in range(args.max_valid_steps):
            try:
                b = next(itr)
            except StopIteration:
                break
            b = _cp_slice(b, cp)
            src, tgt = b["src_tokens"].to(device), b["target"].to(device)
            logits, _ = model(src)
            loss = ops.cross_entropy(logits.reshape(-1, logits.shape[-1]), tgt.reshape(-1), task.tokenizer.pad_id)
            tot += torch.stack([loss.double().reshape(()),
                                torch.tensor(float(b["ntokens"]), dtype=torch.float64, device=device)])
    if hasattr(itr, "close"):
        itr.close()
    if D.is_dist():
        dist.all_reduce(tot)
        tot /= tp                       # the ranks of a tensor-parallel group computed the same loss
    model.train(was_training)
    bits = float(tot[0] / tot[1].clamp_min(1)) / math.log(2)
    return {"loss": round(bits, 3), "ppl": round(2 ** bits, 2), "ntokens": int(tot[1])}


def main(argv=None) -> int:
    args = parse_with_preset(train_parser(), argv)
    device = setup_runtime(args)
    rank, world = D.rank(), D.world()
    if args.criterion != "cross_entropy":
        raise SystemExit("training runs the cross_entropy criterion (the evaluation criterions are for validate)")
    task = build_task(args)
    ds = task.load_dataset("train")
    model, family = build_model(args, task, device)
    optim = OptimConfig(lr=args.lr[0], betas=args.adam_betas, eps=args.adam_eps, weight_decay=args.weight_decay,
                        clip_norm=args.clip_norm, warmup_updates=args.warmup_updates,
                        total_num_update=args.total_num_update, end_learning_rate=args.end_learning_rate,
                        power=args.power)
    tp = args.model_parallel_size
    cp = args.context_parallel_size
    if tp > 1 and cp > 1:
        raise SystemExit("tensor and context parallelism cannot be combined")
    if tp > 1 and family != "yoco":
        raise SystemExit("tensor-parallel training is implemented for YOCO (the LLaMA baseline's output layer returns "
                         "only this rank's vocabulary slice, as in the reference, which evaluation handles)")
    rep = cp if cp > 1 else tp                # consecutive ranks that hold one model replica
    dp = world // rep
    comm = args.comm if (dp > 1 and device.type == "cuda" and rep == 1) else "nccl"
    overlap, transport = exchange_schedule(dp, comm, args.overlap, args.transport)
    if tp > 1:
        overlap, transport = False, "sm"
    graph = bool(args.cuda_graph) and device.type == "cuda" and rep == 1
    trainer = Trainer(model, optim, device=device, comm=comm, graph_step=graph,
                      overlap=overlap, transport=transport, partition=args.partition, pad_idx=task.tokenizer.pad_id,
                      chunk=args.zero_chunk, zero_sharding=args.zero_sharding)
    if cp > 1:
        if family != "yoco":
            raise SystemExit("context parallelism is implemented for YOCO")
        if args.tokens_per_sample % cp:
            raise SystemExit("--tokens-per-sample must be divisible by --context-parallel-size")
    # data shards are per data-parallel replica; the ranks of one context- / tensor-parallel group read the same
    # batches
    itr = task.get_batch_iterator(ds, max_sentences=args.batch_size, seed=args.seed, num_shards=dp,
                                  shard_id=rank // rep)
    restore = os.path.join(args.save_dir, args.restore_file)
    if os.path.exists(part_path(restore)) and not args.reset_optimizer:
        ck = load_checkpoint(restore, model, trainer, reset_lr_scheduler=args.reset_lr_scheduler)
        its = (ck.get("extra_state") or {}).get("train_iterator")
        if its and not args.reset_dataloader and hasattr(itr, "load_state_dict") and len(its) == world:
            itr.load_state_dict(its[rank])
        if rank == 0:
            print(f"| loaded checkpoint {restore} (num_updates {trainer.num_updates()})", flush=True)
    if rank == 0:
        n = sum(p.numel() for p in model.parameters())
        print(f"| model {args.arch} ({family}), params {n:,}, world {world}, comm {comm}, device {device}", flush=True)

    t_start = time.perf_counter()
    while args.max_update <= 0 or trainer.num_updates() < args.max_update:
        batches = [_cp_slice(next(itr), cp) for _ in range(args.update_freq)]
        trainer.train_step(batches if args.update_freq > 1 else batches[0])
        nu = trainer.num_updates()
        if nu % args.log_interval == 0:
            stats = trainer.log_stats()
            stats["num_updates"] = nu
            stats["lr"] = trainer.sched.lr_for(nu)
            stats["train_wall"] = round(time.perf_counter() - t_start, 1)
            line = format_log(stats, fmt=args.log_format)
            if rank == 0 and line:
                print(line, flush=True)
        if (not args.disable_validation and args.validate_interval_updates > 0
                and nu % args.validate_interval_updates == 0):
            trainer.sync_params()          # lazily gathered parameters current before evaluating
            v = validate_lm(model, task, args, device, rank, world, rep, cp, tp)
            if v is not None and rank == 0:
                print(f"valid on '{args.valid_subset}' subset | loss {v['loss']} | ppl {v['ppl']} | "
                      f"num_updates {nu}", flush=True)
        if args.save_model_only and args.save_interval_updates > 0 and nu % args.save_interval_updates == 0:
            _save_model_only(args, model, nu, trainer.rank)
        elif not args.no_save and args.save_interval_updates > 0 and nu % args.save_interval_updates == 0:
            states = _gather_iterator_states(itr)
            save_checkpoint(os.path.join(args.save_dir, f"checkpoint_1_{nu}.pt"), model, trainer,
                            extra_state={"train_iterator": states})
            if trainer.rank == 0:            # data-parallel rank 0 of every tensor-parallel slice
                import shutil
                shutil.copyfile(part_path(os.path.join(args.save_dir, f"checkpoint_1_{nu}.pt")),
                                part_path(os.path.join(args.save_dir, "checkpoint_last.pt")))
            D.barrier()                      # every part written before any rank prunes
            if rank == 0:
                prune_interval_checkpoints(args.save_dir, args.keep_interval_updates)
    trainer.pending.check(block=True)
    if not args.disable_validation and args.validate_interval_updates <= 0:
        trainer.sync_params()
        v = validate_lm(model, task, args, device, rank, world, rep, cp, tp)
        if v is not None and rank == 0:
            print(f"valid on '{args.valid_subset}' subset | loss {v['loss']} | ppl {v['ppl']} | "
                  f"num_updates {trainer.num_updates()}", flush=True)
    if args.save_model_only:
        _save_model_only(args, model, trainer.num_updates(), trainer.rank)
    elif not args.no_save:
        states = _gather_iterator_states(itr)
        save_checkpoint(os.path.join(args.save_dir, "checkpoint_last.pt"), model, trainer,
                        extra_state={"train_iterator": states})
    if hasattr(itr, "close"):
        itr.close()
    trainer.release_graph()
    D.barrier()
    D.destroy()
    return 0


def cli_main():
    sys.exit(main())


if __name__ == "__main__":
    cli_main()
