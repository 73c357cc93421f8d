"""The training step: forward, loss, backward, gradient reduction, clip, sharded Adam, parameter exchange.

Reference: the patched fairseq ``Trainer.train_step`` (yoco/tasks/trainer_nosync.py:219-305) with ZeRO-1 fast path
(yoco/tasks/zero1_fast.py) and the CUDA-graphed decoder layers (yoco/models/decoder/layer_graphs.py). Differences by
design:

* no host syncs at all inside an update: the gradient normaliser ``world / sample_size``, the clip coefficient, the
  learning rate and Adam's bias corrections are device tensors; the non-finite / cross-rank-inconsistent grad-norm
  abort is raised from pinned host memory at the latest one update later (``PendingChecks``);
* ``graph_step=True`` captures the WHOLE update (forward, backward, gradient reduction, Adam, all-gather) as one CUDA
  graph after warm-up; each update is then an input copy, a hyper-parameter copy and one graph launch.
"""
from __future__ import annotations

import contextlib
import math
from typing import Dict, Optional

import torch
import torch.distributed as dist

from .. import ops
from ..parallel import dist as D
from ..parallel.zero import FlatParams, ZeroOptimizer
from ..utils.faults import PendingChecks, grad_norm_consistent
from ..utils.tracing import phase
from .metrics import DeviceMeters
from .schedule import PolynomialDecaySchedule


class _CommHooks:
    """Per-bucket callbacks the model calls: before(b) ahead of bucket b's first forward use, ready(b) from the
    gradient hook that fires once bucket b's backward is complete."""

    def __init__(self, p2p):
        self.p2p = p2p

    def before(self, b: int):
        self.p2p.wait_gather(b)

    def ready(self, b: int):
        self.p2p.bucket_ready(b)


class Trainer:
    def __init__(self, model: torch.nn.Module, optim_cfg, *, device, comm: str = "nccl",
                 pad_idx: int = 1, graph_step: bool = False, group=None, check_consistency: bool = True,
                 overlap=False, partition: str = "even", criterion=None, transport: str = "sm",
                 chunk: Optional[int] = None, zero_sharding: str = "os"):
        """overlap: False (the serial exchange after backward), True (gradients pushed to their owners per layer
        bucket during backward and parameters per bucket ahead of the next forward) or "grads" (gradients per bucket
        during backward, parameters by the fused Adam + push after the update)."""
        from ..parallel import tp as TP
        overlap_params = "bucketed"
        if overlap == "grads":
            overlap, overlap_params = True, "fused"
            if transport == "gemm":
                overlap = False              # the GEMMs already deliver the gradients during backward
        overlap = bool(overlap)
        self.tp = TP.tp_size()
        if self.tp > 1:
            # tensor x data parallelism: ZeRO shards over the data-parallel group (ranks holding the same TP slice);
            # the model's TP layers carry their own collectives; the module path runs without a captured graph
            if group is None:
                group = TP.dp_group()
            if comm == "fused" or transport == "gemm" or overlap:
                raise ValueError("tensor-parallel training runs the NCCL data-parallel exchange (--comm nccl)")
            graph_step = False
        self.model = model
        self.device = torch.device(device)
        self.cfg = optim_cfg
        self.pad_idx = pad_idx
        if group is not None:
            self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        else:
            self.rank, self.world = D.rank(), D.world()
        self.group = group
        if zero_sharding not in ("os", "none"):
            raise ValueError(f"unknown zero_sharding {zero_sharding!r}")
        replicas = 1
        if zero_sharding == "none":
            # fairseq's plain data parallelism: every rank keeps all optimizer state; gradients all-reduced
            replicas, comm, overlap = self.world, "nccl", False
        if comm == "fused" and self.world > 1 and not D.single_node(group):
            # CUDA IPC peer mappings exist only between the GPUs of one node: across nodes the NCCL path runs
            comm, overlap = "nccl", False
            if transport == "gemm":
                transport = "sm"
        p2p = None
        if comm == "fused" and self.world > 1 and self.device.type == "cuda":
            from ..parallel.p2p import PeerComm
            p2p = PeerComm(group)
        fw, fr = (1, 0) if replicas > 1 else (self.world, self.rank)
        self.flat = FlatParams(model.named_parameters(), fw, fr, self.device,
                               dtype=next(model.parameters()).dtype, allocator=p2p.alloc if p2p else None,
                               partition=partition, chunk=chunk)
        self.flat.direct_grads = self.device.type == "cuda" and ops.get_backend() == "native"
        self.zero = ZeroOptimizer(self.flat, optim_cfg, comm=comm, group=group, replicas=replicas)
        import os as _os0
        if (_os0.environ.get("FYB_GEMM_SQ", "1") == "1" and self.world == 1 and self.flat.direct_grads
                and TP.tp_size() == 1):
            # one GPU: the gradient norm from the weight-gradient GEMMs' epilogues (no second pass over 6.9 GB;
            # 70.2 vs 71.2 ms per YOCO-3B update); FYB_GEMM_SQ=0 takes the separate pass
            self.flat.enable_grad_sq()
        if self.tp > 1:
            self.zero.set_tensor_parallel(TP.tp_group(), TP.tp_rank(), TP.is_sharded)
        self.zero.p2p = p2p
        if transport not in ("sm", "ce", "gemm", "pull"):
            raise ValueError(f"unknown transport {transport!r}")
        if transport == "pull":
            overlap = False                  # the all-gather runs inside the forward GEMMs instead
        self.overlap = p2p is not None and overlap and hasattr(model, "param_buckets")
        if p2p is not None and transport == "gemm":
            # gradients: the weight-gradient GEMMs store at the owners; parameters: pushed per layer bucket ahead of
            # the next forward (overlap) or by the fused Adam + push after the update (serial)
            if not self.flat.direct_grads:
                raise ValueError("transport 'gemm' needs the native kernels (weight gradients written by the GEMM)")
            if len(list(model.named_parameters(remove_duplicate=False))) != len(list(model.parameters())):
                raise ValueError("transport 'gemm' stores each weight gradient at its owners once: tied weights "
                                 "(share_input_output_embed) need transport 'sm' or 'ce'")
            p2p.setup_scatter(self.flat)
            if self.overlap:
                p2p.setup_buckets(self.flat, model.param_buckets(), transport="sm", grads="scatter")
        elif p2p is not None and transport == "pull":
            # parameters: the all-gather fused into the consuming forward GEMMs (gemm_gather); gradients: the
            # serial P2P reduce-to-owner after backward
            if not self.flat.direct_grads:
                raise ValueError("transport 'pull' needs the native kernels (the gather-GEMM)")
            p2p.setup_pull(self.flat, model)
        elif self.overlap:
            p2p.setup_buckets(self.flat, model.param_buckets(), transport=transport, params=overlap_params)
        self.sched = PolynomialDecaySchedule(optim_cfg.lr, optim_cfg.warmup_updates, optim_cfg.total_num_update,
                                             optim_cfg.end_learning_rate, optim_cfg.power)
        self.pending = PendingChecks(self.device.type == "cuda")
        self.meters = DeviceMeters(self.device)
        self.check_consistency = check_consistency
        self.graph_step = graph_step and self.device.type == "cuda"
        self._graph = None
        self._static: Dict[str, torch.Tensor] = {}
        self._graph_out = None
        self.vocab = None
        import os as _os
        self._timeline_on = _os.environ.get("FYB_TIMELINE", "0") == "1" and self.device.type == "cuda"
        self._timeline = None
        self.criterion = criterion

    # ------------------------------------------------------------------------------------------------------------
    def num_updates(self) -> int:
        return self.zero.num_updates

    def _to_device(self, batch):
        """Pinned host -> device copies without blocking (yoco/tasks/trainer_nosync.py:67-88)."""
        out = {}
        for k in ("src_tokens", "target"):
            t = batch[k]
            if t.device.type == "cpu" and self.device.type == "cuda":
                if not t.is_pinned():
                    t = t.pin_memory()
                t = t.to(self.device, non_blocking=True)
            out[k] = t
        return out

    def _mark(self, name):
        """Device-event timeline of one update (FYB_TIMELINE=1, eager mode): phase boundaries on the compute stream."""
        if self._timeline is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self._timeline.append((name, ev))

    def timeline(self):
        """[(phase, ms)] of the last update recorded with FYB_TIMELINE=1."""
        if not self._timeline:
            return []
        torch.cuda.synchronize()
        out = []
        for (n0, e0), (n1, e1) in zip(self._timeline, self._timeline[1:]):
            out.append((f"{n0}->{n1}", e0.elapsed_time(e1)))
        return out

    def _forward_backward(self, src, tgt, first: bool = True, last: bool = True):
        self._mark("start")
        with phase("forward"):
            if self.overlap:
                self.zero.p2p.start_gather()
                logits, _ = self.model(src, comm_hooks=_CommHooks(self.zero.p2p))
            else:
                logits, _ = self.model(src)
            V = logits.shape[-1]
            if self.criterion is not None:
                loss = self.criterion(logits, tgt)
            else:
                loss = ops.cross_entropy(logits.view(-1, V), tgt.reshape(-1), self.pad_idx)
        self._mark("forward")
        with phase("backward"):
            loss.backward()
        self._mark("backward")
        return loss.detach()

    def measure_without_exchange(self, on: bool = True):
        """Measurement only: run updates with no cross-rank exchange at all (no gradient reduction, parameter
        all-gather, statistics or grad-norm all-reduce; weight gradients stay local), so that the step time of the
        same work minus its communication can be timed and the exposed communication derived. Ranks' parameters
        diverge: use it after the real measurements. Drops the captured graph (the update is captured again)."""
        self.release_graph()
        self.zero.skip_exchange = on
        if on:
            self._saved_modes = (self.flat.scatter, self.check_consistency, self.overlap, self.flat.pull)
            self.flat.scatter = None
            self.flat.pull = None            # no pulls inside the GEMMs
            self.check_consistency = False
            self.overlap = False             # no per-bucket pushes or waits either
        elif getattr(self, "_saved_modes", None) is not None:
            self.flat.scatter, self.check_consistency, self.overlap, self.flat.pull = self._saved_modes
            self._saved_modes = None

    def _reduce_stats(self, loss_sum, sample_size):
        stats = torch.stack([loss_sum.float().reshape(()), sample_size.float().reshape(())])
        if self.world > 1 and not self.zero.skip_exchange:
            if self.zero.p2p is not None:
                stats = self.zero.p2p.all_reduce_vector(stats)
            else:
                dist.all_reduce(stats, group=self.group)
        return stats[0], stats[1]

    def _device_update(self, srcs, tgts, ntok):
        """All device work of one update (capturable): returns (loss_sum, sample_size, grad_norm, consistent).
        srcs / tgts: the update's micro-batches (``update_freq`` of them); gradients accumulate across them."""
        self._timeline = [] if (self._timeline_on and not self.graph_step) else None
        self.flat.begin_update()
        loss = None
        n = len(srcs)
        for i, (src, tgt) in enumerate(zip(srcs, tgts)):
            self.flat.begin_microbatch(i == 0, i == n - 1)
            li = self._forward_backward(src, tgt, first=i == 0, last=i == n - 1)
            loss = li if loss is None else loss + li
        with phase("reduce-grads"):
            self.flat.collect_grads()          # p.grad -> slot for gradients not written there by a native op
            loss_all, ss_all = self._reduce_stats(loss, ntok)
            sq = self.zero.reduce_grads()
        self._mark("reduced")
        with phase("optimizer"):
            gnorm = self.zero.device_step(ss_all, sq)
        self._mark("optimizer")
        if self.check_consistency:
            reduce = self.zero.p2p.all_reduce_vector if self.zero.p2p is not None else None
            consistent = grad_norm_consistent(gnorm, self.rank, self.world, self.group, reduce=reduce)
        else:
            consistent = torch.isfinite(gnorm)
        return loss_all, ss_all, gnorm, consistent

    def train_step(self, batch) -> torch.Tensor:
        """One update over a batch, or over a list of micro-batches (``--update-freq``); returns the (device) summed
        loss over ranks without waiting for it."""
        self.pending.check(block=False)
        self.model.train()
        batches = batch if isinstance(batch, (list, tuple)) else [batch]
        if self.overlap and len(batches) > 1:
            raise ValueError("overlapped communication hands gradients to their owners during backward; "
                             "use update_freq 1 with it (or overlap=False)")
        devs = [self._to_device(b) for b in batches]
        ntokens = sum(int(b["ntokens"]) for b in batches)
        nsent = sum(int(b.get("nsentences", b["src_tokens"].shape[0])) for b in batches)
        ntok = torch.as_tensor(float(ntokens), dtype=torch.float32)
        lr = self.sched.lr_for(self.num_updates())
        srcs, tgts = [d["src_tokens"] for d in devs], [d["target"] for d in devs]
        if self.graph_step:
            out = self._graph_update(srcs, tgts, ntok, lr)
        else:
            ntok_d = ntok.to(self.device, non_blocking=True) if self.device.type == "cuda" else ntok
            self.zero.prepare(lr)
            out = self._device_update(srcs, tgts, ntok_d)
        loss_all, ss_all, gnorm, consistent = out
        self.pending.check(block=True)
        self.pending.arm(torch.isfinite(gnorm), consistent)
        self.zero.finish()
        self.meters.update(loss_all, ss_all, ntokens * self.world, nsent * self.world, gnorm, self.cfg.clip_norm)
        return loss_all

    # ------------------------------------------------------------------------------------------------------------
    def _graph_update(self, srcs, tgts, ntok, lr):
        st = self._static
        if self._graph is not None and ([tuple(s.shape) for s in srcs] != [tuple(s.shape) for s in st["src"]]):
            self._graph, self._graph_out = None, None          # new batch geometry: capture again
        if self._graph is None:
            st["src"] = [torch.empty_like(s) for s in srcs]
            st["tgt"] = [torch.empty_like(t) for t in tgts]
            st["ntok"] = torch.zeros((), dtype=torch.float32, device=self.device)
        for d, s in zip(st["src"], srcs):
            d.copy_(s, non_blocking=True)
        for d, t in zip(st["tgt"], tgts):
            d.copy_(t, non_blocking=True)
        st["ntok"].copy_(ntok, non_blocking=True)
        self.zero.prepare(lr)
        if self._graph is None:
            # one eager update on a side stream (allocator warm-up, lazy init), then capture the next one
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                out = self._device_update(st["src"], st["tgt"], st["ntok"])
            torch.cuda.current_stream().wait_stream(s)
            self._graph = "warm"
            return out
        if self._graph == "warm":
            g = torch.cuda.CUDAGraph()
            torch.cuda.synchronize()
            with torch.cuda.graph(g):
                self._graph_out = self._device_update(st["src"], st["tgt"], st["ntok"])
            self._graph = g
        self._graph.replay()
        return tuple(t.clone() for t in self._graph_out)

    def sync_params(self):
        """Make every rank's full parameter copy current (the overlapped path gathers lazily at the next update)."""
        if getattr(self.flat, "pull", None) is not None and self.zero.p2p is not None:
            # the pulled weights are current only where a GEMM read them: gather everything
            fp = self.flat
            self.zero.p2p.all_gather(fp.flat, fp.seg, fp.used, chunk=fp.chunk)
            return
        if getattr(self, "overlap", False):
            p2p = self.zero.p2p
            p2p.start_gather()
            for b in range(p2p.nb):
                p2p.wait_gather(b)
            p2p.finish_reduce_reset()

    def release_graph(self):
        """Drop the captured update (must happen before the process group is destroyed)."""
        self._graph = None
        self._graph_out = None

    # ------------------------------------------------------------------------------------------------------------
    def log_stats(self):
        """Flush the device meters (the one host read per log interval) and surface any device-side error word
        (a bounded wait that ran out inside a kernel, a failed bounds check) as an exception."""
        stats = self.meters.flush()
        if self.device.type == "cuda" and ops.get_backend() == "native":
            from ..utils.faults import DeviceStatus
            DeviceStatus.native().raise_if_set()
        return stats
