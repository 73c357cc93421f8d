"""Host logic of the pull exchange (the ZeRO all-gather fused into the consuming forward GEMMs), on CPU: which
weights a forward GEMM pulls, that each is pulled once per update, and that the optimizer step then pushes only the
rest and passes the barrier instead of the full all-gather."""
import torch

from faster_yoco_b200.config import OptimConfig, build_args
from faster_yoco_b200.models.yoco import YOCO
from faster_yoco_b200.parallel.zero import FlatParams, ZeroOptimizer


def _flat(world=2, rank=0, partition="cyclic"):
    torch.manual_seed(0)
    model = YOCO(build_args("yoco_tiny", max_seq_len=64))
    fp = FlatParams(model.named_parameters(), world, rank, "cpu", dtype=torch.float32, partition=partition,
                    chunk=1024)
    return model, fp


def _pull_ids(model, fp):
    from faster_yoco_b200.parallel.p2p import pull_weight_ids
    return pull_weight_ids(fp, model)


def test_pull_args_once_per_update():
    model, fp = _flat()
    ids = _pull_ids(model, fp)
    assert ids, "the model has GEMM weights"
    fp.pull = {"peers": torch.zeros(2, dtype=torch.int64), "ids": ids}
    w = next(e.param for e in fp.entries if id(e.param) in ids)
    a = fp.pull_args(w)
    assert a is not None
    flat, peers, seg, chunk, rank = a
    assert flat is fp.flat and seg == fp.seg and chunk == fp.chunk and rank == fp.rank
    assert fp.pull_args(w) is None                  # already pulled this update (backward GEMMs read it locally)
    norm = next(e.param for e in fp.entries if e.param.dim() == 1)
    assert fp.pull_args(norm) is None               # not a GEMM weight: pushed after the optimizer step
    fp.begin_update()
    assert fp.pull_args(w) is not None              # the next update pulls it again


def test_embeddings_are_not_pulled():
    model, fp = _flat()
    ids = _pull_ids(model, fp)
    assert id(model.embed_tokens.weight) not in ids
    assert id(model.output_projection.weight) in ids or \
        model.output_projection.weight is model.embed_tokens.weight
    assert all(e.param.dim() == 2 for e in fp.entries if id(e.param) in ids)
    # tied input / output embedding: the shared weight is looked up first, so it is pushed, not pulled
    torch.manual_seed(0)
    tied = YOCO(build_args("yoco_tiny", max_seq_len=64, share_input_output_embed=True))
    ftied = FlatParams(tied.named_parameters(), 2, 0, "cpu", dtype=torch.float32)
    assert id(tied.embed_tokens.weight) not in _pull_ids(tied, ftied)


class _FakePeers:
    buckets = None

    def __init__(self):
        self.calls = []

    def push_rest(self):
        self.calls.append("push_rest")

    def all_gather(self, *a, **k):
        self.calls.append("all_gather")


def test_optimizer_pushes_only_the_rest_in_pull_mode():
    model, fp = _flat(world=2, rank=0)
    zero = ZeroOptimizer(fp, OptimConfig(), comm="fused")
    zero.p2p = _FakePeers()
    fp.pull = {"peers": torch.zeros(2, dtype=torch.int64), "ids": _pull_ids(model, fp)}
    zero.all_gather_params()
    assert zero.p2p.calls == ["push_rest"]
    fp.pull = None
    zero.all_gather_params()
    assert zero.p2p.calls == ["push_rest", "all_gather"]
