"""Process-group plumbing: one process per GPU, torch.distributed over NCCL (gloo on CPU)."""
from __future__ import annotations

import datetime
import os
from typing import Optional

import torch
import torch.distributed as dist


def env_rank() -> int:
    return int(os.environ.get("RANK", "0"))


def env_world() -> int:
    return int(os.environ.get("WORLD_SIZE", "1"))


def env_local_rank() -> int:
    return int(os.environ.get("LOCAL_RANK", "0"))


def single_node(group=None) -> bool:
    """True when every rank of `group` (default: all) runs on this node: torch.distributed.run's LOCAL_WORLD_SIZE
    covers the whole group. Peer-memory (CUDA IPC) collectives need it; without the variable one node is assumed."""
    local = os.environ.get("LOCAL_WORLD_SIZE")
    if local is None:
        return True
    size = dist.get_world_size(group) if dist.is_initialized() else env_world()
    return int(local) >= size and int(local) >= env_world()


def init(backend: Optional[str] = None, timeout_s: float = 600.0) -> int:
    """Initialise the default process group if WORLD_SIZE > 1; returns this rank's CUDA device index (or -1)."""
    dev = -1
    if torch.cuda.is_available():
        dev = env_local_rank() % max(torch.cuda.device_count(), 1)
        torch.cuda.set_device(dev)
    if env_world() > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        kw = dict(backend=backend, timeout=datetime.timedelta(seconds=timeout_s))
        if backend == "nccl" and dev >= 0:
            kw["device_id"] = torch.device("cuda", dev)
        dist.init_process_group(**kw)
    return dev


def is_dist() -> bool:
    return dist.is_available() and dist.is_initialized()


def rank() -> int:
    return dist.get_rank() if is_dist() else 0


def world() -> int:
    return dist.get_world_size() if is_dist() else 1


def barrier():
    if is_dist():
        if dist.get_backend() == "nccl":
            dist.barrier(device_ids=[torch.cuda.current_device()])
        else:
            dist.barrier()


def all_reduce_max(x: float, device=None) -> float:
    if not is_dist():
        return x
    dev = device if device is not None else (torch.device("cuda", torch.cuda.current_device())
                                             if dist.get_backend() == "nccl" else torch.device("cpu"))
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def all_gather_object(obj) -> list:
    """Every rank's ``obj`` (picklable), in rank order; ``[obj]`` without a process group."""
    if not is_dist():
        return [obj]
    out = [None] * dist.get_world_size()
    dist.all_gather_object(out, obj)
    return out


def destroy():
    if is_dist():
        dist.destroy_process_group()
