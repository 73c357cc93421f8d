"""Failure detection without host syncs.

``PendingChecks`` is the deferred-abort of the reference (yoco/tasks/trainer_nosync.py:40-64,133-142): the checks are
computed on the GPU, copied to pinned host memory without blocking, and raised as ``FloatingPointError`` once the copy
has landed -- at the latest before the next update's optimizer step.

``DeviceStatus`` reads the error word that the native kernels with bounded waits write (a wait that runs out of
iterations records where it gave up and returns instead of hanging the GPU).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class PendingChecks:
    def __init__(self, use_cuda: bool):
        self.use_cuda = use_cuda
        self.host = torch.zeros(2, dtype=torch.bool, pin_memory=use_cuda)
        self.event = None
        self.armed = False

    def arm(self, finite: torch.Tensor, consistent: torch.Tensor):
        flags = torch.stack([finite.reshape(()), consistent.reshape(())])
        self.host.copy_(flags, non_blocking=self.use_cuda)
        if self.use_cuda:
            self.event = torch.cuda.Event()
            self.event.record()
        self.armed = True

    def check(self, block: bool):
        if not self.armed:
            return
        if self.event is not None:
            if not block and not self.event.query():
                return
            self.event.synchronize()
        self.armed = False
        finite, consistent = bool(self.host[0]), bool(self.host[1])
        if not consistent:
            raise FloatingPointError("Fatal error: gradients are inconsistent between workers.")
        if not finite:
            raise FloatingPointError("gradients are Nan/Inf")


def grad_norm_consistent(grad_norm: torch.Tensor, rank: int, world: int, group=None, reduce=None) -> torch.Tensor:
    """Trainer._check_grad_norms as a device bool: every rank's norm equal to rank 0's within 1e-6 relative.
    `reduce` (optional) sums a small fp32 vector over ranks (the peer-memory mailbox); default NCCL/gloo."""
    if world == 1:
        return torch.isfinite(grad_norm).reshape(())
    buf = torch.zeros(world, dtype=torch.float32, device=grad_norm.device)
    buf[rank] = grad_norm.float()
    if reduce is not None:
        buf = reduce(buf)
    else:
        dist.all_reduce(buf, group=group)
    return torch.isfinite(buf).all() & ((buf - buf[0]).abs().max() / (buf[0] + 1e-6) < 1e-6)


class DeviceStatus:
    """Error word written by kernels with bounded waits: 0 = ok; otherwise (code << 16) | site."""

    CODES = {1: "peer flag wait timed out", 2: "mbarrier wait timed out", 3: "bounds check failed",
             4: "layout check failed"}

    def __init__(self, device=None, word: torch.Tensor = None):
        """word: the extension's status tensor (``_C.status()``, device memory the kernels write); a private zero
        word when the extension is not in use (CPU)."""
        if word is None:
            word = torch.zeros(4, dtype=torch.int32, device=device)
        self.word = word

    @classmethod
    def native(cls):
        from .. import ops
        return cls(word=ops._C().status())

    def value(self) -> int:
        return int(self.word[0].item())

    def raise_if_set(self):
        w = self.word.cpu().tolist()
        if w[0] != 0:
            code = w[0] >> 16
            raise RuntimeError(f"device status {w[0]:#x}: {self.CODES.get(code, 'unknown')} (site {w[0] & 0xffff},"
                               f" detail {w[1:]})")

    def clear(self):
        self.word.zero_()
