"""ZeRO-1 / ZeRO-2 data parallelism over one flat, owner-partitioned parameter buffer.

Partition (``FlatParams(partition=...)``): "even" (default) cuts the model-ordered flat buffer into equal contiguous
segments, so every owner sends and receives the same bytes; "greedy" is fairscale OSS's rule -- whole parameters in
model order, each to the rank with the smallest running element total (yoco/tasks/zero1_fast.py:52-75 replicates it
for the reference's fast path). Every rank holds the same layout: ``flat[r*seg:(r+1)*seg]`` is owner r's segment,
each parameter a view at a 128-byte aligned offset. Gradients live in a second buffer with the same layout, so
"reduce to owner" is a reduce-scatter of equal segments, and the parameter exchange after the step is an all-gather
of equal segments (in place).

Per update (reference call stack yoco/tasks/trainer_nosync.py:219-305 and zero1_fast.py:139-235):

1. gradients are reduced to their owner, averaged over ranks, BF16 (comm backend ``nccl``: reduce-scatter; ``fused``:
   the P2P reduce kernel of :mod:`faster_yoco_b200.parallel.p2p`, FP32 rank-order sum);
2. ``factor = world / sample_size``; grad norm = factor * sqrt(sum over owners of ||g_owned||^2) (one scalar
   all-reduce); ``factor *= min(1, clip / (norm + 1e-6))``;
3. the owner runs Adam on its FP32 master shard with ``g32 = float(g16) * factor`` and writes the BF16 parameter into
   its segment;
4. every rank receives every segment (all-gather: NCCL, or -- ``fused`` -- the same kernel as step 3 also stores each
   new BF16 value into every peer's buffer over NVLink, or per-layer pushes overlapped with the next forward).
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence

import torch
import torch.distributed as dist

from . import dist as D

ALIGN = 64          # elements (128 bytes of bf16): every parameter view starts 128-byte aligned
CYCLIC_CHUNK = 1 << 18   # elements per chunk of the block-cyclic owner map (512 KB of bf16)


# Measured exchange schedule per GPU count (YOCO-3B, 2,048 tokens per GPU, one node), used by overlap / transport
# "auto": world -> (overlap, transport). 2 and 4 GPUs: gradients pushed by the copy engines per layer bucket during
# backward, parameters by the fused Adam + push (2 GPUs 58.5 ms / update against 60.3 ms with copy-engine pushes of
# both and 61.2 ms serial; 4 GPUs 57.9 against 59.5 ms serial). 8 GPUs and other counts: the serial exchange (P2P
# reduce-to-owner after backward, then the fused Adam + push; 61.5 ms at 8 GPUs against 65.0 ms for the copy-engine
# gradient pushes, which reach only ~210 GB/s in aggregate to 7 peers).
AUTO_SCHEDULE = {2: ("grads", "ce"), 4: ("grads", "ce")}


def exchange_schedule(world: int, comm: str, overlap="auto", transport="auto"):
    """(overlap, transport) for :class:`faster_yoco_b200.train.trainer.Trainer` from the command-line values.
    overlap: "auto", "0" / "1" (or a bool) or "grads"; transport: "auto", "sm", "ce", "gemm" or "pull". "auto" picks
    the measured schedule of this GPU count (AUTO_SCHEDULE) for the peer-memory exchange; an explicit transport
    whose exchange is built differently (gemm, pull) keeps the serial schedule."""
    flag = str(overlap).lower()
    if flag not in ("auto", "grads", "0", "1", "true", "false", "yes", "no", "on", "off"):
        raise ValueError(f"overlap must be auto, 0, 1 or grads, not {overlap!r}")
    if transport not in ("auto", "sm", "ce", "gemm", "pull"):
        raise ValueError(f"unknown transport {transport!r}")
    plan = AUTO_SCHEDULE.get(world) if comm == "fused" else None
    if flag == "auto":
        if plan is not None and transport in ("auto", plan[1]):
            overlap = plan[0]
        else:
            overlap = False
    elif flag == "grads":
        overlap = "grads"
    else:
        overlap = flag in ("1", "true", "yes", "on")
    if transport == "auto":
        transport = plan[1] if plan is not None else "sm"
    return overlap, transport


def greedy_partition(sizes: Sequence[int], world: int) -> List[int]:
    """Owner of each parameter: next parameter to the rank with the smallest running total (ties: lowest rank)."""
    totals = [0] * world
    owners = []
    for n in sizes:
        r = totals.index(min(totals))
        owners.append(r)
        totals[r] += n
    return owners


def _round_up(n: int, a: int) -> int:
    return (n + a - 1) // a * a


@dataclass
class Entry:
    param: torch.nn.Parameter
    name: str
    owner: int
    offset: int        # element offset into the flat buffer (global, includes owner * seg)
    numel: int
    shape: torch.Size


class FlatParams:
    """The flat BF16 parameter buffer + flat gradient buffer; model parameters become views of it."""

    def __init__(self, named_params, world: int, rank: int, device, dtype=torch.bfloat16, allocator=None,
                 partition: str = "even", chunk: Optional[int] = None):
        """allocator(name, numel, dtype) -> tensor: where the flat buffers live (peer-shared memory for the fused
        NVLink collectives); default torch.zeros on `device`.

        partition:
          "greedy" -- fairscale OSS: whole parameters, each to the rank with the smallest running total; a rank's
                      parameters sit in its own segment (the reference's layout, zero1_fast.py:52-75).
          "even"   -- parameters laid out in model order and the flat buffer cut into `world` equal contiguous
                      segments, so one large parameter (the 308M-element embedding) spreads over all owners and
                      every rank sends and receives the same bytes. The optimizer math is elementwise, so the
                      partition changes no result; checkpoints store per-parameter state either way.
          "cyclic" -- parameters laid out in model order, the flat buffer cut into chunks of ``chunk`` elements
                      (default 256 Ki) dealt to the ranks in turn: rank r owns chunks r, r + world, ... . Every
                      large weight is spread over all owners, so an exchange that runs layer by layer during the
                      backward pass (the GEMM-fused reduce-scatter) keeps every rank's NVLink port busy instead of
                      one owner's. An owner's optimizer state is its owned chunks in order (local index c)."""
        named = [(n, p) for n, p in named_params if p.requires_grad]
        self.world, self.rank, self.device, self.dtype = world, rank, torch.device(device), dtype
        self.partition = partition
        self.chunk = 0                     # 0: contiguous owner segments
        placed = []
        if partition == "greedy":
            owners = greedy_partition([p.numel() for _, p in named], world)
            fill = [0] * world
            for (name, p), r in zip(named, owners):
                placed.append((name, p, r, fill[r]))
                fill[r] = _round_up(fill[r] + p.numel(), ALIGN)
            self.seg = max(_round_up(max(fill), 1024), 1024)
            self.used = fill                                 # used (aligned) length of each owner's segment
        elif partition == "even":
            off = 0
            for name, p in named:
                placed.append((name, p, None, off))
                off = _round_up(off + p.numel(), ALIGN)
            self.seg = max(_round_up((off + world - 1) // world, 1024), 1024)
            placed = [(n, p, min(o // self.seg, world - 1), o - min(o // self.seg, world - 1) * self.seg)
                      for n, p, _, o in placed]
            self.used = [max(0, min(self.seg, off - r * self.seg)) for r in range(world)]
        elif partition == "cyclic":
            c = _round_up(int(chunk or CYCLIC_CHUNK), ALIGN)
            off = 0
            for name, p in named:
                placed.append((name, p, None, off))
                off = _round_up(off + p.numel(), ALIGN)
            span = c * world
            self.chunk = c
            self.seg = max(_round_up(off, span), span) // world
            placed = [(n, p, self.owner_of(o), o - self.owner_of(o) * self.seg) for n, p, _, o in placed]
            self.used = [self.seg] * world
        else:
            raise ValueError(f"unknown partition {partition!r}")
        if allocator is None:
            self.flat = torch.zeros(world * self.seg, dtype=dtype, device=self.device)
            self.grad_flat = torch.zeros(world * self.seg, dtype=dtype, device=self.device)
        else:
            self.flat = allocator("param", world * self.seg, dtype)
            self.grad_flat = allocator("grad", world * self.seg, dtype)
        self.entries: List[Entry] = []
        self.by_param: Dict[int, Entry] = {}
        with torch.no_grad():
            for name, p, r, off in placed:
                g_off = r * self.seg + off
                view = self.flat[g_off:g_off + p.numel()].view_as(p)
                view.copy_(p.data.to(dtype))
                p.data = view
                e = Entry(p, name, r, g_off, p.numel(), p.shape)
                self.entries.append(e)
                self.by_param[id(p)] = e
        for e in self.entries:
            e.param._fyb_flat = self                                  # lets ops find the gradient slot
        self.buckets: List[List[Entry]] = []
        self.direct_grads = False          # native ops write weight gradients straight into their slots
        self.accumulate = False            # later micro-batches of an update add into the slots
        self._written = set()
        # GEMM-fused reduce-scatter (set by PeerComm.setup_scatter): weight-gradient GEMMs of an update's last
        # micro-batch store each element at its owner (own slot or the owner's staging slot for this rank)
        self.scatter = None                # device int64 [world]: every rank's staging buffer address
        self.scatter_now = True            # the current micro-batch is the update's last one
        self._scattered = set()
        self._sparse = set()               # scattered by row (only the rows of tokens in the batch)
        # one-GPU gradient norm from the weight-gradient GEMMs (enable_grad_sq): the GEMMs of the update's last
        # micro-batch write sum-of-squares partials of their bf16 output, so only the other gradients need a pass
        self.sq_mode = False
        self.sq_buf = None
        self.sq_used = 0
        self._sq_covered = set()
        self._sq_region = {}               # id(p) -> (start, end) of p's partials in sq_buf this update
        self._sq_chunks = {}               # covered set -> device table of the other gradients' chunks
        # parameter all-gather fused into the consuming forward GEMMs (PeerComm.setup_pull): the weights in
        # pull["ids"] are pulled from their owners by the first K-major GEMM that reads them in an update
        self.pull = None                   # {"peers": device int64 [world] replica addresses, "ids": set of id(p)}
        self._pulled = set()

    # ---------------------------------------------------------------------------------------------------------
    def owner_of(self, x: int) -> int:
        """Owner rank of flat element x."""
        return (x // self.chunk) % self.world if self.chunk else x // self.seg

    def local_of(self, x: int) -> int:
        """Index of flat element x in its owner's optimizer state."""
        if self.chunk:
            return (x // (self.chunk * self.world)) * self.chunk + x % self.chunk
        return x - (x // self.seg) * self.seg

    def owned(self, rank: Optional[int] = None) -> slice:
        """This owner's contiguous segment (contiguous layouts only)."""
        if self.chunk:
            raise RuntimeError("the block-cyclic layout has no contiguous owned segment (use owned_view)")
        r = self.rank if rank is None else rank
        return slice(r * self.seg, r * self.seg + self.seg)

    def owned_view(self, buf: torch.Tensor, rank: Optional[int] = None) -> torch.Tensor:
        """The owned elements of a flat buffer in local order: a contiguous [seg] slice, or in the block-cyclic
        layout a strided [seg / chunk, chunk] view whose row-major order is the local order."""
        r = self.rank if rank is None else rank
        if self.chunk:
            return buf.view(-1, self.world, self.chunk)[:, r, :]
        return buf[r * self.seg:(r + 1) * self.seg]

    def param_segment(self, rank: Optional[int] = None) -> torch.Tensor:
        return self.owned_view(self.flat, rank)

    def grad_segment(self, rank: Optional[int] = None) -> torch.Tensor:
        return self.owned_view(self.grad_flat, rank)

    def to_owner_major(self, buf: torch.Tensor) -> torch.Tensor:
        """A flat buffer rearranged as [world, seg] (row r = rank r's owned elements in local order): itself in the
        contiguous layouts, a permuted copy in the block-cyclic one."""
        if self.chunk:
            return buf.view(-1, self.world, self.chunk).transpose(0, 1).reshape(self.world, self.seg)
        return buf.view(self.world, self.seg)

    def from_owner_major(self, buf: torch.Tensor, owner_major: torch.Tensor):
        """Inverse of to_owner_major: write [world, seg] data back into the flat buffer."""
        if self.chunk:
            buf.view(-1, self.world, self.chunk).copy_(owner_major.view(self.world, -1, self.chunk).transpose(0, 1))
        elif owner_major.data_ptr() != buf.data_ptr():
            buf.copy_(owner_major.view(-1))

    def owner_ranges(self, e: "Entry"):
        """[(global offset, count, owner)] pieces of one parameter, cut at owner boundaries (segment or chunk)."""
        step = self.chunk or self.seg
        out, lo, hi = [], e.offset, e.offset + e.numel
        while lo < hi:
            cut = min(hi, (lo // step + 1) * step)
            out.append((lo, cut - lo, self.owner_of(lo)))
            lo = cut
        return out

    def grad_view(self, p) -> torch.Tensor:
        """A fresh view of p's gradient slot (fresh so autograd's AccumulateGrad adopts it without a copy)."""
        e = self.by_param[id(p)]
        return self.grad_flat[e.offset:e.offset + e.numel].view(e.shape)

    def claim_grad(self, p):
        """Slot for p's weight gradient from a native backward: (view, accumulate-into-it)."""
        if id(p) in self._scattered:
            raise RuntimeError("a weight whose gradient was already stored at its owners got a second gradient "
                               "producer (tied weights): the GEMM-fused reduce-scatter cannot accumulate it")
        acc = self.accumulate or id(p) in self._written
        self._written.add(id(p))
        if id(p) in self._sq_covered:
            # a second gradient producer of one weight (tied weights: the output projection's GEMM, then the
            # embedding backward): the first GEMM's sum-of-squares partials no longer describe the slot, so they are
            # cleared and the slot is counted by the pass over uncovered gradients instead
            self._sq_covered.discard(id(p))
            a, b = self._sq_region.pop(id(p), (0, 0))
            if b > a:
                self.sq_buf[a:b].zero_()
        return self.grad_view(p), acc

    def scatter_target(self, p):
        """Staging addresses when p's weight gradient is to be stored at its owners by the GEMM (GEMM-fused
        reduce-scatter on, last micro-batch of the update), else None. Marks p as delivered to its owners."""
        if self.scatter is None or not self.scatter_now:
            return None
        self._scattered.add(id(p))
        return self.scatter

    def sparse_target(self, p):
        """Like scatter_target, for a producer that stores only some rows at the owners (the embedding): the owners
        keep the rest of these staging regions zero (PeerComm.reduce_scattered)."""
        bases = self.scatter_target(p)
        if bases is not None:
            self._sparse.add(id(p))
        return bases

    def scattered(self) -> frozenset:
        return frozenset(self._scattered)

    def enable_grad_sq(self, slots: int = 1 << 21):
        self.sq_mode = True
        self.sq_buf = torch.zeros(slots, dtype=torch.float32, device=self.device)

    def sq_partials(self, p) -> Optional[torch.Tensor]:
        """The free part of the partials buffer when p's weight-gradient GEMM should produce its sum of squares
        (sum-of-squares mode, last micro-batch, no owner scatter), else None. Marks p as covered."""
        if not self.sq_mode or not self.scatter_now or self.scatter is not None:
            return None
        self._sq_covered.add(id(p))
        return self.sq_buf[self.sq_used:]

    def sq_commit(self, p, count: int):
        """Record that p's GEMM wrote `count` partials at the free part of sq_buf."""
        self._sq_region[id(p)] = (self.sq_used, self.sq_used + count)
        self.sq_used += count

    def grad_sq_total(self) -> torch.Tensor:
        """Sum of squares of the whole (bf16) gradient buffer: the GEMM partials of this update plus one pass over
        every gradient no GEMM covered (device tensor [1])."""
        from .. import ops
        key = frozenset(self._sq_covered)
        chunks = self._sq_chunks.get(key)
        if chunks is None:
            if self.device.type == "cuda" and torch.cuda.is_current_stream_capturing():
                raise RuntimeError("gradient norm: the set of GEMM-covered weights changed under capture")
            rows = []
            for e in self.entries:
                if id(e.param) not in key:
                    for a in range(e.offset, e.offset + e.numel, 1 << 16):
                        rows.append([a, min(1 << 16, e.offset + e.numel - a)])
            chunks = torch.tensor(rows, dtype=torch.int64, device=self.device).view(-1, 2)
            self._sq_chunks[key] = chunks
        rest = ops._C().sq_norm_ranges(self.grad_flat, chunks)     # every gradient no GEMM covered, one launch
        if self.sq_used:
            return (self.sq_buf[:self.sq_used].sum().reshape(1) + rest).reshape(1)
        return rest

    def sparse(self) -> frozenset:
        return frozenset(self._sparse)

    def pull_args(self, p):
        """(flat, peers, seg, chunk, rank) for the gather-GEMM when p's all-gather runs inside the GEMM that consumes
        it and this update has not pulled p yet (marks it pulled), else None."""
        if self.pull is None or id(p) not in self.pull["ids"] or id(p) in self._pulled:
            return None
        self._pulled.add(id(p))
        return self.flat, self.pull["peers"], self.seg, self.chunk, self.rank

    def begin_update(self):
        self.accumulate = False
        self._pulled.clear()
        self._written.clear()
        self._scattered.clear()
        self._sparse.clear()
        self._sq_covered.clear()
        self._sq_region.clear()
        self.sq_used = 0

    def begin_microbatch(self, first: bool, last: bool = True):
        """Gradient accumulation needs no flag: a slot written by an earlier micro-batch of this update is
        accumulated into (claim_grad), autograd accumulates p.grad for the others until collect_grads. With the
        GEMM-fused reduce-scatter, only the last micro-batch's weight-gradient GEMMs store at the owners (adding
        the earlier micro-batches' sums held in the local slots)."""
        self.scatter_now = last

    def collect_grads(self):
        """Move every p.grad into its slot and clear p.grad; slots that no gradient reached this update are zeroed."""
        with torch.no_grad():
            for e in self.entries:
                g = e.param.grad
                slot = self.grad_flat[e.offset:e.offset + e.numel]
                written = id(e.param) in self._written
                if g is not None and id(e.param) in self._scattered:
                    raise RuntimeError(f"{e.name}: gradient from autograd for a weight already stored at its owners")
                if g is None:
                    if not written:
                        slot.zero_()
                elif g.data_ptr() != slot.data_ptr():
                    if written:
                        slot.view(e.shape).add_(g)
                    else:
                        slot.view(e.shape).copy_(g)
                    self._written.add(id(e.param))
                e.param.grad = None

    def make_buckets(self, module_groups: Sequence[Sequence[torch.nn.Parameter]]):
        """Reduction buckets: groups of parameters whose gradients are complete together (one layer each)."""
        self.buckets = [[self.by_param[id(p)] for p in grp if id(p) in self.by_param] for grp in module_groups]
        return self.buckets


def grad_slot(p: torch.Tensor) -> Optional[torch.Tensor]:
    fp = getattr(p, "_fyb_flat", None)
    return fp.grad_view(p) if fp is not None else None


class ZeroOptimizer:
    """Sharded FP32 Adam (apex AdamW expression) over the owner's segment of a :class:`FlatParams`."""

    def __init__(self, flat: FlatParams, optim_cfg, comm: str = "nccl", group=None, replicas: int = 1):
        """replicas > 1: no sharding (``--zero-sharding none``, fairseq's plain data parallelism): ``flat`` is one
        segment holding everything, the gradient buffer is averaged over the `replicas` ranks of `group` and every
        rank runs the full Adam step."""
        self.flat, self.cfg, self.comm, self.group = flat, optim_cfg, comm, group
        self.replicas = replicas
        if replicas > 1 and flat.world != 1:
            raise ValueError("unsharded data parallelism keeps one segment (FlatParams world 1)")
        seg = flat.param_segment()
        self.master = seg.reshape(-1).float().clone()       # local order (a gather in the block-cyclic layout)
        self.exp_avg = torch.zeros_like(self.master)
        self.exp_avg_sq = torch.zeros_like(self.master)
        self.num_updates = 0
        dev = flat.device
        # device-resident hyper-parameters: [lr, bias_correction1, bias_correction2] (written by the host each step)
        self.hyper = torch.zeros(4, dtype=torch.float32, device=dev)
        self._hyper_host = torch.zeros(4, dtype=torch.float32, pin_memory=dev.type == "cuda")
        self.p2p = None
        # serial peer-memory exchange: Adam and the all-gather push as one kernel (FYB_FUSE_ADAM_PUSH=0 runs them
        # as two passes, Adam then push_range, for comparison)
        self.fuse_adam_push = os.environ.get("FYB_FUSE_ADAM_PUSH", "1") != "0"
        # contiguous owner segments: Adam through the 8-elements-per-thread kernel (the Adam + push kernel with no
        # peers; 6.01 vs 5.72 TB/s for the 4-wide kernel over 1 Gi elements); FYB_ADAM8=0 takes the 4-wide kernel.
        # The block-cyclic layout keeps the 4-wide kernel (its owner-map addressing)
        self.adam8 = os.environ.get("FYB_ADAM8", "1") == "1" and flat.chunk == 0
        self.last_grad_norm = None
        # measurement only (Trainer.measure_without_exchange): no cross-rank exchange at all, each rank steps its
        # owned parameters from its own gradients -- the compute-only time of an update, not a training mode
        self.skip_exchange = False
        self.tp_group = None

    def set_tensor_parallel(self, tp_group, tp_rank: int, is_sharded):
        """Tensor x data parallelism: this optimizer shards over the data-parallel group; the global gradient norm
        adds every TP rank's sharded parameters and counts the replicated ones (identical on all TP ranks: norm
        weights) once, so clipping matches TP = 1."""
        fp = self.flat
        self.tp_group, self.tp_rank = tp_group, tp_rank
        rep = [(o, c) for e in fp.entries if not is_sharded(e.param)
               for o, c, r in fp.owner_ranges(e) if r == fp.rank]
        self._rep_pieces = rep
    # ---------------------------------------------------------------------------------------------------------
    def reduce_grads(self):
        """Average the gradient buffer over ranks into each owner's segment (BF16). Returns the owned segment's sum
        of squares when the reduction produced it (fused path), else None."""
        fp = self.flat
        if self.replicas > 1 and not self.skip_exchange:
            g = fp.grad_flat
            if dist.get_backend(self.group) == "nccl":
                dist.all_reduce(g, op=dist.ReduceOp.AVG, group=self.group)
            else:
                dist.all_reduce(g, group=self.group)
                g.div_(self.replicas)
            return None
        if fp.world == 1 or self.skip_exchange:
            return None
        if self.comm == "fused" and self.p2p is not None:
            if self.p2p.buckets is not None:
                return self.p2p.finish_reduce()
            if fp.scatter is not None:
                return self.p2p.reduce_scattered(fp)
            return self.p2p.reduce_to_owner(fp.grad_flat, fp.seg, fp.used[fp.rank], chunk=fp.chunk)
        # library path: reduce-scatter over the owner-major arrangement (the buffer itself when contiguous)
        src = fp.to_owner_major(fp.grad_flat).reshape(-1)
        out = fp.grad_segment() if not fp.chunk else torch.empty(fp.seg, dtype=fp.dtype, device=fp.device)
        if dist.get_backend(self.group) == "nccl":
            dist.reduce_scatter_tensor(out, src, op=dist.ReduceOp.AVG, group=self.group)
        else:
            tmp = torch.empty_like(out)
            dist.reduce_scatter_tensor(tmp, src, op=dist.ReduceOp.SUM, group=self.group)
            out.copy_(tmp / fp.world)
        if fp.chunk:
            fp.grad_segment().copy_(out.view(-1, fp.chunk))
        return None

    def all_gather_params(self):
        fp = self.flat
        if fp.world == 1 or self.skip_exchange:
            return
        if self.comm == "fused" and self.p2p is not None:
            if self.p2p.buckets is not None and self.p2p.params_mode == "bucketed":
                return          # pushed bucket by bucket ahead of the next update's forward (overlapped)
            if fp.pull is not None:
                # the GEMM weights are pulled by their consumers in the next forward; push the rest, then one
                # barrier publishes this owner's update to the pullers
                self.p2p.push_rest()
                return
            self.p2p.all_gather(fp.flat, fp.seg, fp.used, chunk=fp.chunk)
            return
        if not fp.chunk:
            dist.all_gather_into_tensor(fp.flat, fp.param_segment(), group=self.group)
            return
        full = torch.empty(fp.world * fp.seg, dtype=fp.dtype, device=fp.device)
        dist.all_gather_into_tensor(full, fp.param_segment().reshape(-1), group=self.group)
        fp.from_owner_major(fp.flat, full.view(fp.world, fp.seg))

    def prepare(self, lr: float):
        """Host part before an update: learning rate and bias corrections into the device hyper-parameter vector."""
        step = self.num_updates + 1
        b1, b2 = self.cfg.betas
        bc1 = float(torch.tensor(1.0 - b1 ** step, dtype=torch.float32))
        bc2 = float(torch.tensor(1.0 - b2 ** step, dtype=torch.float32))
        h = self._hyper_host
        h[0], h[1], h[2], h[3] = lr, bc1, bc2, float(step)
        self.hyper.copy_(h, non_blocking=True)
        self._lr = lr

    def finish(self):
        self.num_updates += 1

    def device_step(self, sample_size: torch.Tensor, sq: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Clip + Adam + parameter exchange, device work only (capturable). sample_size: device scalar summed
        over ranks; sq: this owner's sum of squares if the reduction already produced it. Returns the grad norm."""
        from .. import ops
        fp = self.flat
        g16 = fp.grad_segment()
        factor = max(fp.world, self.replicas) / torch.where(sample_size > 0, sample_size,
                                                            torch.ones_like(sample_size)).float()
        native = ops.native_on(g16)
        if sq is not None:
            sq = sq.clone()
        elif native and fp.sq_mode and fp.world == 1 and self.replicas == 1 and self.tp_group is None:
            sq = fp.grad_sq_total()
        elif native:
            sq = ops._C().sq_norm(g16.reshape(-1))
        else:
            sq = g16.float().pow(2).sum().reshape(1)
        if self.tp_group is not None and self.tp_rank != 0 and self._rep_pieces:
            # replicated parameters enter the norm once: from TP rank 0 (the reduced gradients are identical there)
            rep = torch.stack([fp.grad_flat[o:o + c].float().pow(2).sum() for o, c in self._rep_pieces]).sum()
            sq = sq - rep.reshape(1)
        if fp.world > 1 and not self.skip_exchange:
            if self.comm == "fused" and self.p2p is not None:
                sq = self.p2p.all_reduce_vector(sq)
            else:
                dist.all_reduce(sq, group=self.group)
        if self.tp_group is not None:
            dist.all_reduce(sq, group=self.tp_group)
        grad_norm = (factor * sq.sqrt()).reshape(())
        clip = self.cfg.clip_norm
        if clip > 0:
            factor = factor * (clip / (grad_norm + 1e-6)).clamp(max=1.0)
        b1, b2 = self.cfg.betas
        seg = fp.param_segment()
        fused_push = (native and fp.world > 1 and self.comm == "fused" and self.p2p is not None
                      and (self.p2p.buckets is None or self.p2p.params_mode == "fused") and self.fuse_adam_push
                      and not self.skip_exchange and fp.pull is None)
        # the kernels address this owner's bf16 gradients / parameters through the owner map: its segment views
        # (contiguous layouts) or the whole flat buffers + the chunk size (block-cyclic)
        g_arg, p_arg = (fp.grad_flat, fp.flat) if fp.chunk else (g16, seg)
        if fused_push:
            # one pass: Adam on this owner's segment + the all-gather push of its new bf16 values to every peer
            ops._C().adam_push(self.master, g_arg, self.exp_avg, self.exp_avg_sq, p_arg, self.hyper,
                               factor.reshape(1).float().contiguous(), float(b1), float(b2), float(self.cfg.eps),
                               float(self.cfg.weight_decay), bool(self.cfg.adamw_mode), self.p2p.peers["param"],
                               0 if fp.chunk else fp.owned().start, fp.rank, fp.chunk)
            self.p2p.barrier()
        elif native and self.adam8:
            # the Adam + push kernel with no peers: the same update, 8 elements per thread
            ops._C().adam_push(self.master, g_arg, self.exp_avg, self.exp_avg_sq, p_arg, self.hyper,
                               factor.reshape(1).float().contiguous(), float(b1), float(b2), float(self.cfg.eps),
                               float(self.cfg.weight_decay), bool(self.cfg.adamw_mode), [p_arg.data_ptr()],
                               0, 0, 0)
        elif native:
            ops._C().adam_step(self.master, g_arg, self.exp_avg, self.exp_avg_sq, p_arg, self.hyper,
                               factor.reshape(1).float().contiguous(), float(b1), float(b2), float(self.cfg.eps),
                               float(self.cfg.weight_decay), bool(self.cfg.adamw_mode), fp.chunk, fp.world,
                               fp.rank)
        else:
            self._torch_adam(g16, seg, factor, self._lr)
        if not fused_push:
            self.all_gather_params()
        self.last_grad_norm = grad_norm
        return grad_norm

    def step(self, sample_size: torch.Tensor, lr: float) -> torch.Tensor:
        self.prepare(lr)
        n = self.device_step(sample_size)
        self.finish()
        return n

    def _torch_adam(self, g16, seg, factor, lr):
        from ..ops import reference as ref
        b1, b2 = self.cfg.betas
        g32 = g16.reshape(-1).float() * factor.float()
        ref.adam_step_(self.master, g32, self.exp_avg, self.exp_avg_sq, lr=lr, beta1=b1, beta2=b2,
                       eps=self.cfg.eps, step=self.num_updates + 1, weight_decay=self.cfg.weight_decay,
                       adamw=self.cfg.adamw_mode)
        seg.copy_(self.master.view(seg.shape).to(seg.dtype))

    # ---------------------------------------------------------------------------------------------------------
    def state_dict(self):
        return {"num_updates": self.num_updates, "master": self.master, "exp_avg": self.exp_avg,
                "exp_avg_sq": self.exp_avg_sq, "seg": self.flat.seg, "rank": self.flat.rank,
                "world": self.flat.world, "chunk": self.flat.chunk}

    def load_state_dict(self, sd):
        if sd["seg"] != self.flat.seg or sd["world"] != self.flat.world or sd.get("chunk", 0) != self.flat.chunk:
            raise ValueError("optimizer shard layout does not match this run (seg/world/chunk differ)")
        self.num_updates = int(sd["num_updates"])
        self.master.copy_(sd["master"])
        self.exp_avg.copy_(sd["exp_avg"])
        self.exp_avg_sq.copy_(sd["exp_avg_sq"])

    def consolidated_state(self):
        """Per-parameter FP32 master / exp_avg / exp_avg_sq gathered on every rank (for a consolidated checkpoint)."""
        fp = self.flat
        shards = {}
        for name, t in (("master", self.master), ("exp_avg", self.exp_avg), ("exp_avg_sq", self.exp_avg_sq)):
            if fp.world > 1:
                full = torch.empty(fp.world * fp.seg, dtype=t.dtype, device=t.device)
                dist.all_gather_into_tensor(full, t, group=self.group)
            else:
                full = t
            if fp.chunk:                      # owner-major -> flat order
                flat_order = torch.empty_like(full)
                fp.from_owner_major(flat_order, full.view(fp.world, fp.seg))
                full = flat_order
            shards[name] = full
        out = {}
        for e in fp.entries:
            out[e.name] = {k: v[e.offset:e.offset + e.numel].view(e.shape).cpu().clone() for k, v in shards.items()}
        return out
