"""GEMM-fused ZeRO reduce-scatter, host side (CPU): where each weight-gradient element is stored, that the owners'
staged sums equal the plain average over ranks, and the push / own tables that complete the exchange."""
import torch

from faster_yoco_b200.ops import reference as ref
from faster_yoco_b200.parallel.zero import FlatParams


def _model():
    torch.manual_seed(0)
    return torch.nn.ModuleDict({
        "emb": torch.nn.Embedding(97, 24),
        "qkv": torch.nn.Linear(24, 72, bias=False),
        "norm": torch.nn.LayerNorm(24, elementwise_affine=True, bias=False),
        "fc": torch.nn.Linear(24, 40, bias=False),
    })


def test_owner_scatter_then_staged_sum_is_the_average():
    world = 4
    m = _model()
    flats = [FlatParams(_model().named_parameters(), world, r, "cpu") for r in range(world)]
    seg = flats[0].seg
    own = [torch.zeros(world * seg, dtype=torch.bfloat16) for _ in range(world)]
    staging = [torch.zeros(world * seg, dtype=torch.bfloat16) for _ in range(world)]
    grads = {}
    for r in range(world):
        g = torch.Generator().manual_seed(10 + r)
        for e in flats[r].entries:
            dw = torch.randn(e.shape, generator=g).to(torch.bfloat16)
            grads[(r, e.name)] = dw
            ref.owner_scatter(dw, e.offset, seg, r, own[r], staging)
    # every entry straddling owners is covered: the staged sum equals the rank-order average
    assert any(len(flats[0].owner_ranges(e)) > 1 for e in flats[0].entries)
    for s in range(world):
        for e in flats[s].entries:
            for lo, n, owner in flats[s].owner_ranges(e):
                if owner != s:
                    continue
                got = ref.staged_owner_sum(own[s], staging[s], s, world, seg, lo, n)
                i0 = lo - e.offset
                acc = torch.zeros(n)
                for r in range(world):
                    acc += grads[(r, e.name)].reshape(-1)[i0:i0 + n].float()
                want = (acc * (1.0 / world)).to(torch.bfloat16)
                assert torch.equal(got, want), (e.name, s)
    del m


class _FakePeers:
    """The table builder of PeerComm without CUDA or a process group."""

    def __init__(self, rank):
        from faster_yoco_b200.parallel.p2p import PeerComm
        self.rank, self.dev, self._scatter_tables = rank, torch.device("cpu"), {}
        self.tables = PeerComm._scatter_tables_for.__get__(self)


def test_scatter_tables_cover_every_piece_once():
    world = 3
    for rank in range(world):
        fp = FlatParams(_model().named_parameters(), world, rank, "cpu")
        fp.scatter = torch.zeros(world, dtype=torch.int64)
        fp.begin_update()
        gemm_written = [e for e in fp.entries if e.name in ("qkv.weight", "fc.weight")]
        for e in gemm_written:
            assert fp.scatter_target(e.param) is fp.scatter
        push, own = _FakePeers(rank).tables(fp)
        pieces = [pc for e in fp.entries for pc in fp.owner_ranges(e)]
        want_own = sorted((o, c) for o, c, r in pieces if r == rank)
        scattered = {id(e.param) for e in gemm_written}
        want_push = sorted((o, c, r) for e in fp.entries if id(e.param) not in scattered
                           for o, c, r in fp.owner_ranges(e) if r != rank)
        assert sorted(map(tuple, own.tolist())) == want_own
        assert sorted(map(tuple, push.tolist())) == want_push


def test_scatter_target_only_on_last_microbatch():
    fp = FlatParams(_model().named_parameters(), 2, 0, "cpu")
    p = fp.entries[1].param
    assert fp.scatter_target(p) is None                 # scatter off
    fp.scatter = torch.zeros(2, dtype=torch.int64)
    fp.begin_update()
    fp.begin_microbatch(True, False)
    assert fp.scatter_target(p) is None and fp.scattered() == frozenset()
    fp.begin_microbatch(False, True)
    assert fp.scatter_target(p) is fp.scatter and fp.scattered() == frozenset({id(p)})
    # a weight whose gradient already went to its owners must not also arrive through autograd
    p.grad = torch.zeros_like(p)
    try:
        fp.collect_grads()
    except RuntimeError as e:
        assert "owners" in str(e)
    else:
        raise AssertionError("collect_grads accepted an autograd gradient for a scattered weight")
