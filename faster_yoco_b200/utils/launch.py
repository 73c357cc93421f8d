"""Multi-process launcher for tests and tools: run `fn(rank, world, *args)` in `world` processes that form a
torch.distributed group (gloo on CPU, nccl with one GPU per rank), rendezvous on 127.0.0.1."""
from __future__ import annotations

import datetime
import os
import socket
import traceback

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _entry(rank, world, port, backend, fn, args, errq, timeout_s):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        kw = {}
        if backend == "nccl":
            torch.cuda.set_device(rank)
            kw["device_id"] = torch.device("cuda", rank)
        dist.init_process_group(backend, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=timeout_s), **kw)
        fn(rank, world, *args)
        if dist.is_initialized():          # fn may have torn the group down itself (the CLI entry points do)
            dist.barrier()
    except Exception:
        errq.put((rank, traceback.format_exc()))
        raise
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def run_ranks(fn, world: int, *args, backend: str = "gloo", timeout_s: float = 120.0):
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = free_port()
    procs = [ctx.Process(target=_entry, args=(r, world, port, backend, fn, args, errq, timeout_s))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout_s + 60)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    if errs or alive or any(p.exitcode != 0 for p in procs):
        raise RuntimeError(f"ranks failed: exitcodes={[p.exitcode for p in procs]} errors={errs}")
