"""GEMM-fused ZeRO reduce-scatter, host side (CPU): where each weight-gradient element is stored, that the owners'
staged sums equal the plain average over ranks, and the push / own tables that complete the exchange."""
import pytest
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


@pytest.mark.parametrize("partition", ["even", "cyclic"])
def test_scatter_tables_cover_every_piece_once(partition):
    world = 3
    for rank in range(world):
        fp = FlatParams(_model().named_parameters(), world, rank, "cpu", partition=partition, chunk=256)
        fp.scatter = torch.zeros(world, dtype=torch.int64)
        fp.begin_update()
        gemm_written = [e for e in fp.entries if e.name in ("qkv.weight", "fc.weight")]
        for e in gemm_written:
            assert fp.scatter_target(e.param) is fp.scatter
        push = _FakePeers(rank).tables(fp)
        scattered = {id(e.param) for e in gemm_written}
        want_push = sorted((o, c, r) for e in fp.entries if id(e.param) not in scattered
                           for o, c, r in fp.owner_ranges(e) if r != rank)
        assert sorted(map(tuple, push.tolist())) == want_push
        # together with the GEMM-written weights, every piece another rank owns reaches it exactly once
        sent = sorted(map(tuple, push.tolist())) + sorted(
            (o, c, r) for e in gemm_written for o, c, r in fp.owner_ranges(e) if r != rank)
        assert sorted(sent) == sorted((o, c, r) for e in fp.entries for o, c, r in fp.owner_ranges(e) if r != rank)


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


def test_cyclic_owner_map_is_consistent():
    world, chunk = 3, 128
    fp = FlatParams(_model().named_parameters(), world, 1, "cpu", partition="cyclic", chunk=chunk)
    assert fp.chunk == chunk and fp.seg % chunk == 0 and fp.flat.numel() == world * fp.seg
    n = fp.flat.numel()
    x = torch.arange(n)
    owner = torch.tensor([fp.owner_of(int(i)) for i in x])
    local = torch.tensor([fp.local_of(int(i)) for i in x])
    # every (owner, local) pair is hit exactly once and local indices cover [0, seg) per owner
    for r in range(world):
        assert sorted(local[owner == r].tolist()) == list(range(fp.seg))
    # the owned view lists this rank's elements in local order
    probe = x.to(torch.float64)
    for r in range(world):
        v = fp.owned_view(probe, r).reshape(-1)
        assert torch.equal(local[v.long()], torch.arange(fp.seg)) and bool((owner[v.long()] == r).all())
    # owner-major arrangement and back
    om = fp.to_owner_major(probe)
    assert om.shape == (world, fp.seg)
    back = torch.empty_like(probe)
    fp.from_owner_major(back, om)
    assert torch.equal(back, probe)
    # pieces never cross a chunk and carry their owner; every large weight has pieces at every owner
    for e in fp.entries:
        pcs = fp.owner_ranges(e)
        assert sum(c for _, c, _ in pcs) == e.numel
        for o, c, r in pcs:
            assert o // chunk == (o + c - 1) // chunk and fp.owner_of(o) == r
        if e.numel >= world * chunk * 2:
            assert {r for _, _, r in pcs} == set(range(world))


def test_owner_scatter_cyclic_staging_layout():
    """The cyclic layout's scatter destination: owner (x // chunk) % world, slot position local(x)."""
    world, chunk, rank = 4, 64, 2
    fp = FlatParams(_model().named_parameters(), world, rank, "cpu", partition="cyclic", chunk=chunk)
    seg = fp.seg
    e = max(fp.entries, key=lambda t: t.numel)
    dw = torch.randn(e.shape).to(torch.bfloat16)
    own = torch.zeros(world * seg, dtype=torch.bfloat16)
    staging = [torch.zeros(world * seg, dtype=torch.bfloat16) for _ in range(world)]
    flat = dw.reshape(-1)
    for i in range(flat.numel()):
        x = e.offset + i
        o = fp.owner_of(x)
        if o == rank:
            own[x] = flat[i]
        else:
            staging[o][rank * seg + fp.local_of(x)] = flat[i]
    # the owner-side view: owner o reads slot `rank` in local order; the elements it owns of this weight match
    for o in range(world):
        if o == rank:
            continue
        for off, c, r in fp.owner_ranges(e):
            if r != o:
                continue
            lo = fp.local_of(off)
            assert torch.equal(staging[o][rank * seg + lo: rank * seg + lo + c], flat[off - e.offset: off - e.offset + c])
