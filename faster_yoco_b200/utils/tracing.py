"""Named ranges for profilers: ``torch.profiler`` ranges always (the reference's ``record_function`` phases
"forward", "backward", "reduce-grads", "clip-grads", "optimizer": yoco/tasks/trainer_nosync.py:268-288,
tasks/gpt.py:154-158) and NVTX ranges when ``FYB_NVTX=1`` or inside :func:`emit_nvtx` (the ``--profile`` switch of the
eval entry, yoco/validate.py:282-285). Both are host-side markers: they add no device work and are legal inside CUDA
graph capture."""
from __future__ import annotations

import contextlib
import os

import torch

_NVTX = os.environ.get("FYB_NVTX", "0") == "1"


@contextlib.contextmanager
def phase(name: str):
    nvtx = _NVTX and torch.cuda.is_available()
    if nvtx:
        torch.cuda.nvtx.range_push(name)
    try:
        with torch.autograd.profiler.record_function(name):
            yield
    finally:
        if nvtx:
            torch.cuda.nvtx.range_pop()


@contextlib.contextmanager
def emit_nvtx(enabled: bool = True):
    """NVTX ranges for every autograd op plus this module's phases (for an external profiler)."""
    global _NVTX
    if not enabled or not torch.cuda.is_available():
        yield
        return
    old, _NVTX = _NVTX, True
    try:
        with torch.autograd.profiler.emit_nvtx():
            yield
    finally:
        _NVTX = old
