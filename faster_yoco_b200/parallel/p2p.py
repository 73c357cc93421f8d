"""NVLink peer-memory communication for ZeRO: CUDA-IPC shared buffers and the fused collectives of ``csrc/comm.cu``.

Each rank ``cudaMalloc``s its flat parameter buffer, flat gradient buffer, a flag array and a small mailbox, exports
IPC handles, and opens every peer's handles once (the reference does the same for its copy-engine path,
yoco/models/decoder/ce_reduce.py:77-98). After that, the collectives of an update are plain kernel launches that
read and write peer memory directly over NVLink / NVSwitch:

* ``reduce_to_owner``: flag barrier (all ranks finished the backward), then the owner's kernel sums its segment of
  every rank's gradient buffer in FP32 rank order, divides by world, writes BF16 in place and returns the segment's
  sum of squares (the grad-norm partial) -- one pass instead of NCCL reduce + scale kernel + norm kernel;
* ``all_gather``: every owner stores its updated segment into every peer's buffer (remote stores run at NVLink speed,
  remote loads do not), then one flag barrier publishes the pushes;
* ``all_reduce_vector``: up to 32 fp32 values summed in rank order through the mailboxes (loss / sample size /
  grad norm) -- no NCCL launch on the update path;
* bucketed overlap (``setup_buckets``): per layer bucket, gradient pieces are pushed to their owners during backward
  and parameters are pushed ahead of the next forward, either by kernels (``transport="sm"``) or by the copy
  engines (``transport="ce"``: one ``cudaMemcpyAsync`` per piece on one stream per peer, arrival published by a
  one-thread release-add on the peer's counter); the owner sums the staged pieces from local memory. With
  ``params="fused"`` only the gradients travel per bucket: the parameters go out with the fused Adam + push after
  the update, as in the serial exchange;
* GEMM-fused reduce-scatter (``setup_scatter`` / ``reduce_scattered``): the weight-gradient GEMMs and the embedding
  backward store their output at the owners' staging slots while backward runs; after it, one push of the remaining
  gradients, one barrier and the owner's local rank-order sum.

Every kernel addresses owned elements through the owner map of the flat buffers (contiguous segments, or the
block-cyclic chunks of ``FlatParams(partition="cyclic")``, ``csrc/common/zero_map.cuh``).

The order in which ranks call these is identical by construction, so one flag slot with a monotonically increasing
epoch serves every barrier. All waits are bounded on the device (a timeout sets the status word read by
:class:`faster_yoco_b200.utils.faults.DeviceStatus`).
"""
from __future__ import annotations

import os
from typing import Dict, List, Optional, Tuple

import torch
import torch.distributed as dist

from .. import ops


def pull_weight_ids(flat, model) -> set:
    """The weights whose all-gather the consuming forward GEMM carries (pull exchange): every 2-D parameter both of
    whose dimensions are multiples of 8 (the shapes the native GEMM takes; others run on the library path, which
    reads the local replica as it is), except embeddings (their forward is a row lookup, not a GEMM; a weight tied
    to one is excluded with it)."""
    embed = {id(p) for n, p in model.named_parameters(remove_duplicate=False) if "embed" in n}
    return {id(e.param) for e in flat.entries
            if e.param.dim() == 2 and id(e.param) not in embed and e.param.shape[0] % 8 == 0
            and e.param.shape[1] % 8 == 0}


def bucket_pieces(flat, groups, rank: int):
    """Per bucket (parameter groups in forward order), the pieces of its parameters cut at owner boundaries:
    (owned, other) with owned[b] = [[flat offset, count], ...] of the pieces `rank` owns (it sums them) and
    other[b] = [[flat offset, count, owner], ...] of the pieces it sends to their owners."""
    owned, other = [], []
    for grp in groups:
        ents = [flat.by_param[id(p)] for p in grp if id(p) in flat.by_param]
        pieces = [pc for e in ents for pc in flat.owner_ranges(e)]
        owned.append([[o, c] for o, c, r in pieces if r == rank])
        other.append([[o, c, r] for o, c, r in pieces if r != rank])
    return owned, other


class PeerComm:
    NSLOTS = 64          # flag slots: 0 = generic barrier, 1..61 = reduction buckets, 63 = gather barrier
    GATHER_SLOT = 63

    def __init__(self, group=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > 8:
            raise ValueError("peer-memory collectives support at most 8 ranks (one NVSwitch domain)")
        self.C = ops._C()
        self.dev = torch.device("cuda", torch.cuda.current_device())
        self._keep: List[torch.Tensor] = []
        self._opened: List[int] = []
        self.flags, self.peer_flags = self.share_bytes(self.NSLOTS * 8 * 4)
        self.box, self.peer_box = self.share_bytes(2 * 8 * 32 * 4)
        self.box_f = self.box.view(torch.float32)
        # device-resident barrier epochs (one per flag slot) and mailbox call counter: graph replays stay correct
        self.counters = torch.zeros(self.NSLOTS + 1, dtype=torch.int32, device=self.dev)
        self.buckets = None
        self.params_mode = "bucketed"
        self.peers: Dict[str, List[int]] = {}
        P = min(2 * torch.cuda.get_device_properties(self.dev).multi_processor_count, 1024)
        self.part = torch.zeros(P, dtype=torch.float32, device=self.dev)
        self.sq = torch.zeros(1, dtype=torch.float32, device=self.dev)
        self._gather_segs: Dict[Tuple, torch.Tensor] = {}

    # ------------------------------------------------------------------------------------------------- buffers
    def share_bytes(self, nbytes: int) -> Tuple[torch.Tensor, List[int]]:
        t, h = self.C.ipc_alloc(int(nbytes))
        handles = [None] * self.world
        dist.all_gather_object(handles, h.tolist(), group=self.group)
        ptrs = []
        for r in range(self.world):
            if r == self.rank:
                ptrs.append(t.data_ptr())
            else:
                p = self.C.ipc_open(torch.tensor(handles[r], dtype=torch.uint8))
                self._opened.append(p)
                ptrs.append(p)
        self._keep.append(t)
        return t, ptrs

    def alloc(self, name: str, numel: int, dtype: torch.dtype) -> torch.Tensor:
        """A shared buffer of `numel` elements; peers' addresses of the same buffer are kept under `name`."""
        esz = torch.empty((), dtype=dtype).element_size()
        t, ptrs = self.share_bytes(numel * esz)
        self.peers[name] = ptrs
        return t.view(dtype)[:numel]

    # ------------------------------------------------------------------------------------------------- collectives
    def barrier(self, slot: int = 0):
        self.C.flag_barrier(self.peer_flags, self.flags, self.counters, self.rank, slot)

    def reduce_to_owner(self, grad_flat: torch.Tensor, seg: int, used: Optional[int] = None,
                        chunk: int = 0) -> torch.Tensor:
        """Average the gradient buffers of all ranks over this rank's owned elements (its segment, or its chunks in
        the block-cyclic layout), in place. Returns their sum of squares after the BF16 rounding (device [1])."""
        n = seg if used is None else used
        self.barrier()
        base = 0 if chunk else self.rank * seg
        self.C.reduce_owner(self.peers["grad"], grad_flat, base, n, self.part, self.sq, chunk, self.rank)
        return self.sq

    def all_gather(self, flat: torch.Tensor, seg: int, used: Optional[List[int]] = None, chunk: int = 0):
        """Push form (remote stores run at NVLink speed where remote loads do not): this rank stores its updated
        elements into every peer's buffer, then one barrier publishes all pushes."""
        n = used[self.rank] if used else seg
        sms = torch.cuda.get_device_properties(self.dev).multi_processor_count
        self.C.push_range(flat, self.peers["param"], 0 if chunk else self.rank * seg, n, self.rank, sms, chunk)
        self.barrier()

    def all_reduce_vector(self, v: torch.Tensor) -> torch.Tensor:
        """Sum of a small fp32 vector over ranks, rank order (returns a new tensor)."""
        v = v.reshape(-1).float().contiguous()
        if v.numel() > 32:
            raise ValueError("all_reduce_vector: at most 32 values")
        box_counter = self.counters[self.NSLOTS:]
        self.C.mailbox_put(self.peer_box, v, self.rank, box_counter)
        self.barrier()
        out = torch.empty_like(v)
        self.C.mailbox_sum(self.box_f, out, self.world, box_counter)
        return out

    # ------------------------------------------------------------------------- GEMM-fused reduce-scatter (serial)
    def setup_scatter(self, flat, push_ctas: Optional[int] = None):
        """Weight-gradient GEMMs store straight at the owners: every rank gets a staging buffer of world x seg
        elements (slot r = rank r's contribution to this rank's segment), and ``flat.scatter`` is set to the device
        list of every rank's staging address, which ``ops.wgrad_into`` passes to the scatter epilogue."""
        if "staging" not in self.peers:
            self.staging = self.alloc("staging", self.world * flat.seg, flat.dtype)
        # slots no rank writes (padding) must read as zero in the owner's sum
        self.staging.zero_()
        torch.cuda.synchronize(self.dev)
        self.flat = flat
        self.scatter_bases = torch.tensor(self.peers["staging"], dtype=torch.int64, device=self.dev)
        flat.scatter = self.scatter_bases
        sms = torch.cuda.get_device_properties(self.dev).multi_processor_count
        self.scatter_push_ctas = push_ctas or sms
        self.scatter_red_ctas = min(2 * sms, self.part.numel())
        self._sarrive, self._peer_sarrive = self.share_bytes(self.NSLOTS * 4)
        self._scatter_tables: Dict[object, torch.Tensor] = {}
        dist.barrier(group=self.group)      # every rank's staging is zeroed before any peer can store into it

    def _scatter_tables_for(self, flat) -> torch.Tensor:
        """Pieces of the gradients NOT stored at their owners by a GEMM that other ranks own ([n, 3]: flat offset,
        count, owner). Built on the first (eager) update and reused, so a captured update launches with a fixed
        table."""
        key = flat.scattered()
        t = self._scatter_tables.get(key)
        if t is None:
            if self.dev.type == "cuda" and torch.cuda.is_current_stream_capturing():
                raise RuntimeError("GEMM-fused reduce-scatter: the set of scattered weights changed under capture")
            push = [[o, c, r] for e in flat.entries if id(e.param) not in key
                    for o, c, r in flat.owner_ranges(e) if r != self.rank]
            t = torch.tensor(push, dtype=torch.int64, device=self.dev).view(-1, 3)
            self._scatter_tables[key] = t
        return t

    def reduce_scattered(self, flat) -> torch.Tensor:
        """End of backward with the GEMM-fused reduce-scatter: push the gradients no GEMM delivered (norm weights,
        the embedding, anything autograd produced) to their owners' staging slots, one barrier (every rank's GEMM
        epilogue stores and pushes are done), then the owner sums its owned elements from local memory in rank
        order (its own values + the staging slots; same arithmetic as ``reduce_to_owner``). Returns their sum of
        squares after the BF16 rounding."""
        push = self._scatter_tables_for(flat)
        if push.numel():
            # the arrival counts of this push are not waited on: the barrier below publishes it
            self.C.push_grads(flat.grad_flat, self.peers["staging"], self._peer_sarrive, push, 0, self.rank,
                              flat.seg, self.scatter_push_ctas, flat.chunk)
        self.barrier()
        part = self.part[: self.scatter_red_ctas]
        self.C.reduce_compact(flat.grad_flat, self.staging, flat.used[self.rank], self.world, self.rank, flat.seg,
                              flat.chunk, part, self.scatter_red_ctas)
        self.C.sum_partials(part, self.sq)
        # rows stored sparsely (the embedding): clear them for the next update; peers store again only after the
        # barrier that ends this update's parameter exchange, which this rank reaches after the clear
        zero = self._sparse_table_for(flat)
        if zero.numel():
            self.C.zero_staged(self.staging, zero, self.world, self.rank, flat.seg, self.scatter_push_ctas)
        return self.sq

    def _sparse_table_for(self, flat) -> torch.Tensor:
        """Local ranges [n, 2] (local offset, count) of this owner's pieces of the sparsely scattered weights."""
        key = ("sparse", flat.sparse())
        t = self._scatter_tables.get(key)
        if t is None:
            if self.dev.type == "cuda" and torch.cuda.is_current_stream_capturing():
                raise RuntimeError("GEMM-fused reduce-scatter: the set of sparsely scattered weights changed under "
                                   "capture")
            rows = [[flat.local_of(o), c] for e in flat.entries if id(e.param) in key[1]
                    for o, c, r in flat.owner_ranges(e) if r == self.rank]
            t = torch.tensor(rows, dtype=torch.int64, device=self.dev).view(-1, 2)
            self._scatter_tables[key] = t
        return t

    # ------------------------------------------------------------------------------------ overlapped (bucketed)
    def setup_buckets(self, flat, groups, reduce_ctas: Optional[int] = None, gather_ctas: Optional[int] = None,
                      transport: str = "sm", grads: str = "push", params: str = "bucketed"):
        """groups: parameter lists in FORWARD order (bucket b = groups[b]). Precomputes, per bucket, the ranges this
        rank owns (reduced during backward) and the ranges it must pull from other owners (before forward).

        transport "sm": the pushes are kernels (remote stores from CTAs); "ce": the pushes are cudaMemcpyAsync
        transfers on one stream per peer (the copy engines move the data, so no SM time is taken from the GEMMs of
        the overlapped forward / backward), each followed by a one-thread kernel that publishes the arrival.

        params "bucketed": parameters are pushed bucket by bucket ahead of the next forward (start_gather /
        wait_gather); "fused": only the gradients are exchanged per bucket, the parameters by the fused Adam + push
        kernel after the update (its closing barrier also tells every owner that its staging slots may be written
        again)."""
        if len(groups) > self.NSLOTS - 3:
            raise ValueError("too many buckets")
        if transport not in ("sm", "ce") or grads not in ("push", "scatter") or params not in ("bucketed", "fused"):
            raise ValueError((transport, grads, params))
        self.transport = transport
        self.params_mode = params
        # grads "scatter": the weight-gradient GEMMs store at the owners (setup_scatter), so no bucket pushes
        # gradients; finish_reduce pushes the rest and sums (reduce_scattered)
        self.grads_mode = grads
        reduce_ctas = int(os.environ.get("FYB_REDUCE_CTAS", reduce_ctas or 128))
        gather_ctas = int(os.environ.get("FYB_PUSH_CTAS", gather_ctas or 128))
        self.flat = flat
        own_l, oth_l = bucket_pieces(flat, groups, self.rank)
        owned = [torch.tensor(t, dtype=torch.int64, device=self.dev).view(-1, 2) for t in own_l]
        other = [torch.tensor(t, dtype=torch.int64, device=self.dev).view(-1, 3) for t in oth_l]
        self.buckets = (owned, other)
        self.nb = len(groups)
        # push-based parameter exchange: per-bucket arrival counters (peers add into ours) + local expectations
        self.arrive, self.peer_arrive = self.share_bytes(self.NSLOTS * 4)
        self.expected = torch.zeros(self.NSLOTS, dtype=torch.int32, device=self.dev)
        self.push_ctas = gather_ctas
        # push-based gradient reduction: peers store their pieces of this rank's segment into staging slot [peer]
        if "staging" not in self.peers:
            self.staging = self.alloc("staging", self.world * flat.seg, flat.dtype)
        self.garrive, self.peer_garrive = self.share_bytes(self.NSLOTS * 4)
        self.gexpected = torch.zeros(self.NSLOTS, dtype=torch.int32, device=self.dev)
        self.grad_push_ctas = reduce_ctas
        self.red_ctas, self.gather_ctas = reduce_ctas, gather_ctas
        self.bucket_part = torch.zeros(self.nb, reduce_ctas, dtype=torch.float32, device=self.dev)
        self.stream = torch.cuda.Stream(device=self.dev, priority=-1)
        self.ready_ev = [torch.cuda.Event() for _ in range(self.nb)]
        self.gather_ev = [torch.cuda.Event() for _ in range(self.nb)]
        self.start_ev = torch.cuda.Event()
        self._reduced = [False] * self.nb
        # copy-engine transport: FYB_CE_BUCKET_SUM=1 sums each bucket's staged pieces on the communication stream as
        # soon as every peer's pieces of it have arrived (during backward) instead of all buckets after backward
        self.ce_bucket_sum = transport == "ce" and os.environ.get("FYB_CE_BUCKET_SUM", "0") == "1"
        if transport == "ce":
            # host-side piece lists (byte offsets) and one copy stream per peer
            esz = flat.flat.element_size()
            self.ce_owned = [[(int(o) * esz, int(c) * esz) for o, c in t.tolist()] for t in owned]
            self.ce_other = [[(int(o) * esz, int(c) * esz, int(q)) for o, c, q in t.tolist()] for t in other]
            self.peer_streams = {q: torch.cuda.Stream(device=self.dev) for q in range(self.world) if q != self.rank}
            self.ce_done = torch.cuda.Event()

    # ----------------------------------------------------------------- all-gather fused into the forward GEMMs
    def setup_pull(self, flat, model):
        """The parameter all-gather moves into the consumers: every 2-D weight except embeddings is pulled from its
        owners by the first forward GEMM that reads it (gemm_gather: the GEMM's gather warps copy the rows ahead of
        the tiles); after the optimizer step this rank pushes only the rest (embeddings, norm weights) and passes
        one barrier, which also tells the pullers that its owned rows are final. Best with the block-cyclic owner
        map: a tile column then spans several owners, and pulls from several peers at once run near link speed
        where pulls from one peer do not."""
        ids = pull_weight_ids(flat, model)
        rest = [[o, c] for e in flat.entries if id(e.param) not in ids
                for o, c, r in flat.owner_ranges(e) if r == self.rank]
        self.rest_ranges = torch.tensor(rest, dtype=torch.int64, device=self.dev).view(-1, 2)
        if not hasattr(self, "peer_arrive"):
            self.arrive, self.peer_arrive = self.share_bytes(self.NSLOTS * 4)
        flat.pull = {"peers": torch.tensor(self.peers["param"], dtype=torch.int64, device=self.dev), "ids": ids}
        self.flat = flat

    def push_rest(self):
        """Pull mode, after the optimizer step: push this owner's parameters that no GEMM pulls, then barrier."""
        sms = torch.cuda.get_device_properties(self.dev).multi_processor_count
        if self.rest_ranges.numel():
            self.C.push_bucket(self.flat.flat, self.peers["param"], self.peer_arrive, self.rest_ranges,
                               self.NSLOTS - 2, self.rank, sms)
        self.barrier()

    def _slot_barrier(self, slot: int):
        self.C.flag_barrier(self.peer_flags, self.flags, self.counters, self.rank, slot)

    def _ce_start_gather(self):
        cur = torch.cuda.current_stream(self.dev)
        self.start_ev.record(cur)
        src = self.flat.flat.data_ptr()
        for q, st in self.peer_streams.items():
            dst = self.peers["param"][q]
            with torch.cuda.stream(st):
                st.wait_event(self.start_ev)
                for b in range(self.nb):
                    for o, c in self.ce_owned[b]:
                        self.C.peer_copy(dst + o, src + o, c)
                    self.C.signal_peer(self.peer_arrive[q], b)
        self._reduced = [False] * self.nb

    def _ce_bucket_ready(self, b: int):
        cur = torch.cuda.current_stream(self.dev)
        self.ready_ev[b].record(cur)
        grad = self.flat.grad_flat.data_ptr()
        esz = self.flat.grad_flat.element_size()
        seg_b = self.flat.seg * esz
        for q, st in self.peer_streams.items():
            slot = self.peers["staging"][q] + self.rank * seg_b     # owner q's staging slot for this rank
            with torch.cuda.stream(st):
                st.wait_event(self.ready_ev[b])
                for o, c, owner in self.ce_other[b]:
                    if owner == q:
                        self.C.peer_copy(slot + self.flat.local_of(o // esz) * esz, grad + o, c)
                self.C.signal_peer(self.peer_garrive[q], b)
        if self.ce_bucket_sum:
            # this owner's part of bucket b: wait (bounded) for every peer's pieces, then sum them with its own
            # values, which are final once the bucket's backward is
            owned, _ = self.buckets
            with torch.cuda.stream(self.stream):
                self.stream.wait_event(self.ready_ev[b])
                self.C.wait_arrivals(self.garrive, self.gexpected, b, self.world - 1)
                self.C.reduce_staged(self.flat.grad_flat, self.staging, owned[b], self.world, self.rank,
                                     self.flat.seg, self.bucket_part[b], self.red_ctas, self.flat.chunk)

    def _ce_finish_reduce(self) -> torch.Tensor:
        cur = torch.cuda.current_stream(self.dev)
        for st in self.peer_streams.values():
            cur.wait_stream(st)                    # my pushes are done (staging of peers, gradient buffer reusable)
        if self.ce_bucket_sum:                     # every bucket was summed on the communication stream
            cur.wait_stream(self.stream)
            self.C.sum_partials(self.bucket_part.view(-1), self.sq)
            return self.sq
        for b in range(self.nb):
            self.C.wait_arrivals(self.garrive, self.gexpected, b, self.world - 1)
        owned_all = self._owned_all()
        part = self.bucket_part.view(-1)[: self.red_ctas_all]
        self.C.reduce_staged(self.flat.grad_flat, self.staging, owned_all, self.world, self.rank, self.flat.seg,
                             part, self.red_ctas_all, self.flat.chunk)
        self.C.sum_partials(part, self.sq)
        return self.sq

    def _owned_all(self) -> torch.Tensor:
        if getattr(self, "_owned_all_t", None) is None:
            owned, _ = self.buckets
            rows = torch.cat([t for t in owned if t.numel()], 0) if any(t.numel() for t in owned) else \
                torch.zeros(0, 2, dtype=torch.int64, device=self.dev)
            self._owned_all_t = rows.contiguous()
            sms = torch.cuda.get_device_properties(self.dev).multi_processor_count
            # three CTAs per SM (the staged-sum kernel's register budget): it is latency-bound with fewer loads in
            # flight
            self.red_ctas_all = min(3 * sms, self.bucket_part.numel())
        return self._owned_all_t

    def start_gather(self):
        """Start of an update: this rank pushes the parameters it owns (updated by its previous Adam step), bucket
        by bucket in forward order, into every peer's flat buffer on the communication stream; forward waits per
        bucket for the peers' pushes (wait_gather). Safe: a peer's previous reads of bucket b ended with its
        backward of b, which every owner's reduction of b (hence Adam) waited for."""
        if self.params_mode == "fused":
            self._reduced = [False] * self.nb        # parameters went out with the fused Adam + push
            return
        if self.transport == "ce":
            return self._ce_start_gather()
        cur = torch.cuda.current_stream(self.dev)
        self.start_ev.record(cur)
        owned, _ = self.buckets
        with torch.cuda.stream(self.stream):
            self.stream.wait_event(self.start_ev)
            for b in range(self.nb):
                self.C.push_bucket(self.flat.flat, self.peers["param"], self.peer_arrive, owned[b], b, self.rank,
                                   self.push_ctas)
        self._reduced = [False] * self.nb

    def wait_gather(self, b: int):
        if self.params_mode == "fused":
            return
        inc = (self.world - 1) * (1 if self.transport == "ce" else self.push_ctas)
        self.C.wait_arrivals(self.arrive, self.expected, b, inc)

    def bucket_ready(self, b: int):
        """Bucket b's gradients are final on this rank (called from a gradient hook on the compute stream)."""
        if self._reduced[b]:
            return
        self._reduced[b] = True
        if self.grads_mode == "scatter":
            return
        if self.transport == "ce":
            return self._ce_bucket_ready(b)
        owned, other = self.buckets
        self.ready_ev[b].record(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(self.stream):
            self.stream.wait_event(self.ready_ev[b])
            # push my pieces of bucket b to their owners, wait for every peer's pieces of my part, sum locally
            self.C.push_grads(self.flat.grad_flat, self.peers["staging"], self.peer_garrive, other[b], b, self.rank,
                              self.flat.seg, self.grad_push_ctas, self.flat.chunk)
            self.C.wait_arrivals(self.garrive, self.gexpected, b, (self.world - 1) * self.grad_push_ctas)
            self.C.reduce_staged(self.flat.grad_flat, self.staging, owned[b], self.world, self.rank, self.flat.seg,
                                 self.bucket_part[b], self.red_ctas, self.flat.chunk)

    def finish_reduce(self) -> torch.Tensor:
        """Reduce the buckets no hook reported (in bucket order), join the streams, and return this owner's sum of
        squares of the reduced gradients (fixed summation order)."""
        for b in range(self.nb):
            if not self._reduced[b]:
                self.bucket_ready(b)
        if self.grads_mode == "scatter":
            cur = torch.cuda.current_stream(self.dev)
            cur.wait_stream(self.stream)                 # this update's parameter pushes are done
            for st in getattr(self, "peer_streams", {}).values():
                cur.wait_stream(st)
            return self.reduce_scattered(self.flat)
        if self.transport == "ce":
            return self._ce_finish_reduce()
        torch.cuda.current_stream(self.dev).wait_stream(self.stream)
        self.C.sum_partials(self.bucket_part.view(-1), self.sq)
        return self.sq

    def finish_reduce_reset(self):
        cur = torch.cuda.current_stream(self.dev)
        cur.wait_stream(self.stream)
        for st in getattr(self, "peer_streams", {}).values():
            cur.wait_stream(st)
        self._reduced = [True] * self.nb

    def close(self):
        torch.cuda.synchronize()
        for p in self._opened:
            try:
                self.C.ipc_close(p)
            except Exception:
                pass
        self._opened.clear()
        self._keep.clear()
