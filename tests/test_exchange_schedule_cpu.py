"""Host logic of the exchange schedule: the measured per-GPU-count choice behind overlap / transport "auto", and
which exchange the optimizer step runs for the parameters under each overlap form (CPU, fake peer transport)."""
import pytest
import torch

from faster_yoco_b200.config import OptimConfig, build_args
from faster_yoco_b200.models.yoco import YOCO
from faster_yoco_b200.parallel.zero import FlatParams, ZeroOptimizer


def test_exchange_schedule_auto_and_explicit():
    """The measured exchange schedule behind overlap / transport "auto", and explicit values passed through."""
    from faster_yoco_b200.parallel.zero import AUTO_SCHEDULE, exchange_schedule
    for world, (ov, tr) in AUTO_SCHEDULE.items():
        assert exchange_schedule(world, "fused") == (ov, tr)
        assert exchange_schedule(world, "nccl") == (False, "sm")        # the library path has no peer pushes
    assert exchange_schedule(1, "fused") == (False, "sm")
    assert exchange_schedule(2, "fused", "0", "auto")[0] is False
    assert exchange_schedule(8, "fused", "1", "ce") == (True, "ce")
    assert exchange_schedule(8, "fused", "grads", "ce") == ("grads", "ce")
    assert exchange_schedule(2, "fused", "auto", "pull") == (False, "pull")   # pull carries its own all-gather
    assert exchange_schedule(2, "fused", "auto", "gemm") == (False, "gemm")
    assert exchange_schedule(2, "fused", True, "ce") == (True, "ce")
    for bad in ("grad", "2"):
        with pytest.raises(ValueError):
            exchange_schedule(2, "fused", bad)
    with pytest.raises(ValueError):
        exchange_schedule(2, "fused", "auto", "copy")


class _FakeBuckets:
    """The parts of PeerComm the optimizer step consults, recording the parameter exchanges it asks for."""

    def __init__(self, params_mode):
        self.buckets = ([], [])
        self.params_mode = params_mode
        self.calls = []

    def all_gather(self, *a, **k):
        self.calls.append("all_gather")


def test_parameter_exchange_follows_the_overlap_form():
    torch.manual_seed(0)
    model = YOCO(build_args("yoco_tiny", max_seq_len=64))
    fp = FlatParams(model.named_parameters(), 2, 0, "cpu", dtype=torch.float32)
    zero = ZeroOptimizer(fp, OptimConfig(), comm="fused")
    # overlap 1: the parameters leave per bucket ahead of the next forward, so the step itself sends nothing
    zero.p2p = _FakeBuckets("bucketed")
    zero.all_gather_params()
    assert zero.p2p.calls == []
    # overlap "grads": only the gradients were bucketed; the step sends the parameters (on the GPU the fused
    # Adam + push kernel does it, elsewhere the all-gather after Adam)
    zero.p2p = _FakeBuckets("fused")
    zero.all_gather_params()
    assert zero.p2p.calls == ["all_gather"]


def _model(tied=False):
    torch.manual_seed(0)
    return YOCO(build_args("yoco_tiny", max_seq_len=64, share_input_output_embed=tied))


def test_param_buckets_cover_every_parameter_once():
    """The overlap units (embedding, each layer, shared K/V projection, head) hold every trainable parameter exactly
    once, tied weights included."""
    for tied in (False, True):
        model = _model(tied)
        groups = model.param_buckets()
        ids = [id(p) for g in groups for p in g]
        assert len(ids) == len(set(ids))
        assert set(ids) == {id(p) for p in model.parameters() if p.requires_grad}
        assert groups[0] == [model.embed_tokens.weight]


def test_bucket_pieces_partition_the_flat_buffer():
    """Per bucket, one rank's owned pieces and the pieces it sends cover the bucket's parameters exactly once, every
    piece lies inside one owner's range, and over all ranks every element is summed by exactly one owner."""
    from faster_yoco_b200.parallel.p2p import bucket_pieces
    for partition, chunk in (("even", None), ("greedy", None), ("cyclic", 512)):
        for world in (2, 4):
            model = _model()
            groups = model.param_buckets()
            fps = [FlatParams(model.named_parameters(), world, r, "cpu", dtype=torch.float32, partition=partition,
                              chunk=chunk) for r in range(world)]
            summed = torch.zeros(world * fps[0].seg, dtype=torch.int32)
            for rank, fp in enumerate(fps):
                owned, other = bucket_pieces(fp, groups, rank)
                assert len(owned) == len(other) == len(groups)
                for b, grp in enumerate(groups):
                    cover = torch.zeros(world * fp.seg, dtype=torch.int32)
                    for o, c in owned[b]:
                        assert fp.owner_of(o) == rank and fp.owner_of(o + c - 1) == rank
                        cover[o:o + c] += 1
                        summed[o:o + c] += 1
                    for o, c, q in other[b]:
                        assert q != rank and fp.owner_of(o) == q and fp.owner_of(o + c - 1) == q
                        # a sent piece lands contiguously in the owner's staging slot (at its local offsets)
                        assert fp.local_of(o + c - 1) - fp.local_of(o) == c - 1
                        cover[o:o + c] += 1
                    want = torch.zeros_like(cover)
                    for p in grp:
                        e = fp.by_param[id(p)]
                        want[e.offset:e.offset + e.numel] = 1
                    assert torch.equal(cover, want), (partition, world, rank, b)
            used = torch.zeros_like(summed)
            for e in fps[0].entries:
                used[e.offset:e.offset + e.numel] = 1
            assert torch.equal(summed, used), (partition, world)


class _RecordingPeers:
    """Stand-in for PeerComm in the overlapped schedule on one CPU process: records the calls the trainer and the
    model's communication hooks make; the vector all-reduce adds a second rank with the same values."""

    def __init__(self, nb, params_mode):
        self.buckets = ([None] * nb, [None] * nb)
        self.nb = nb
        self.params_mode = params_mode
        self.calls = []

    def start_gather(self):
        self.calls.append(("start_gather",))

    def wait_gather(self, b):
        self.calls.append(("before", b))

    def bucket_ready(self, b):
        self.calls.append(("ready", b))

    def finish_reduce(self):
        self.calls.append(("finish_reduce",))
        return None

    def all_reduce_vector(self, v):
        return v.reshape(-1).float() * 2

    def all_gather(self, *a, **k):
        self.calls.append(("all_gather",))


def test_overlapped_schedule_call_order():
    """One update of the overlapped exchange (host side): the forward waits for each bucket's parameters in forward
    order, every bucket but the embedding reports its gradients from a hook in reverse order during backward, the
    reduction finishes after the last report, and the parameters are exchanged after Adam only in the gradient-only
    form (the bucketed form pushes them ahead of the next forward instead)."""
    from faster_yoco_b200.train.trainer import Trainer
    cfg = OptimConfig(lr=3e-4, warmup_updates=0, total_num_update=10)
    for params_mode in ("fused", "bucketed"):
        model = _model()
        nb = len(model.param_buckets())
        tr = Trainer(model, cfg, device="cpu")
        fp = FlatParams(model.named_parameters(), 2, 0, "cpu", dtype=torch.float32)     # rank 0 of 2
        tr.flat, tr.zero = fp, ZeroOptimizer(fp, cfg, comm="fused")
        peers = _RecordingPeers(nb, params_mode)
        tr.zero.p2p, tr.overlap, tr.world, tr.check_consistency = peers, True, 2, False
        ids = torch.randint(0, 1024, (2, 65), generator=torch.Generator().manual_seed(0))
        loss = tr.train_step({"src_tokens": ids[:, :-1].contiguous(), "target": ids[:, 1:].contiguous(),
                              "ntokens": 128, "nsentences": 2})
        assert torch.isfinite(loss)
        calls = peers.calls
        assert calls[0] == ("start_gather",)
        before = [c[1] for c in calls if c[0] == "before"]
        ready = [c[1] for c in calls if c[0] == "ready"]
        assert before == list(range(nb))
        assert ready == list(range(nb - 1, 0, -1))          # the head first; the embedding (bucket 0) has no hook
        fin = calls.index(("finish_reduce",))
        assert fin > max(i for i, c in enumerate(calls) if c[0] == "ready")
        gathers = [i for i, c in enumerate(calls) if c == ("all_gather",)]
        assert gathers == ([len(calls) - 1] if params_mode == "fused" else [])
        assert gathers == [] or gathers[0] > fin
