"""GEMM-fused ZeRO reduce-scatter on the GPU: the weight-gradient GEMM whose epilogue stores every element at its
owner, against the plain GEMM + the host-side oracle of where each element goes (one GPU, four ranks' staging
buffers emulated in local memory: the kernel only sees addresses), and 2-GPU training against the serial exchange."""
import math
import os

import pytest
import torch

from faster_yoco_b200 import ops
from faster_yoco_b200.ops import reference as ref

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("chunk", [0, 1024])
@pytest.mark.parametrize("M,N,T,acc", [(200, 96, 256, False), (200, 96, 256, True), (128, 128, 8192, False),
                                       (128, 128, 8192, True), (1024, 3072, 2048, False), (24, 3072, 2048, True)])
def test_gemm_scatter_stores_at_owners(M, N, T, acc, chunk):
    ops.set_backend("native")
    C = ops._C()
    dev = torch.device("cuda", 0)
    world, rank, x0 = 4, 1, 3000
    numel = M * N
    seg = int(math.ceil((x0 + numel) / 3 / 1024)) * 1024          # the slot spans owners 0, 1 and 2
    if chunk:
        seg = int(math.ceil((x0 + numel) / (world * chunk))) * chunk   # chunks dealt to all four owners
    g = torch.Generator(device=dev).manual_seed(M + N + T)
    grad_flat = torch.randn(world * seg, generator=g, device=dev).to(torch.bfloat16)
    staging = [torch.zeros(world * seg, dtype=torch.bfloat16, device=dev) for _ in range(world)]
    bases = torch.tensor([t.data_ptr() for t in staging], dtype=torch.int64, device=dev)
    dy = torch.randn(T, M, generator=g, device=dev).to(torch.bfloat16)
    x = torch.randn(T, N, generator=g, device=dev).to(torch.bfloat16)
    slot = grad_flat[x0:x0 + numel].view(M, N)
    prev = slot.clone()
    want = ops.gemm(dy, x, a_mn_major=True, b_mn_major=True, out=torch.empty(M, N, dtype=torch.bfloat16, device=dev),
                    residual=prev if acc else None)
    own_exp = grad_flat.clone()
    stag_exp = [t.clone() for t in staging]
    ref.owner_scatter(want, x0, seg, rank, own_exp, stag_exp, chunk)
    for _ in range(2):                                             # a second call stores the same values
        if acc:
            slot.copy_(prev)
        C.gemm_scatter(dy, x, slot, acc, grad_flat, bases, seg, rank, chunk)
        torch.cuda.synchronize()
        # this rank's buffer changes only where it owns the slot (elsewhere the slot keeps its earlier contents,
        # which with accumulation are the earlier micro-batches' sums)
        assert torch.equal(grad_flat, own_exp)
        for q in range(world):
            assert torch.equal(staging[q], stag_exp[q]), q
    assert int(C.status()[0].item()) == 0
    # and the GEMM itself against fp32
    r = dy.float().t() @ x.float() + (prev.float() if acc else 0)
    assert ((want.float() - r).abs().max() / r.abs().max()).item() < 2e-2


def _ptrs(ts):
    return [t.data_ptr() for t in ts]


@pytest.mark.parametrize("chunk", [0, 512])
def test_zero_kernels_owner_map_one_gpu(chunk):
    """The exchange kernels under both owner maps, with every rank's buffer emulated in this GPU's memory (a kernel
    sees only addresses): reduce-to-owner, push all-gather, Adam, Adam + push, the gradient push to staging slots
    and the staged owner sum (whole segment, and over a table of owned pieces), each against a PyTorch oracle."""
    ops.set_backend("native")
    C = ops._C()
    dev = torch.device("cuda", 0)
    world, rank = 4, 2
    seg = 8 * 512 if chunk else 8 * 512 + 256
    n = world * seg
    g = torch.Generator(device=dev).manual_seed(7 + chunk)
    x = torch.arange(n, device=dev)
    owner, local = ref.zero_owner_local(x, seg, chunk, world)
    mine = owner == rank
    flat_of_local = torch.empty(seg, dtype=torch.int64, device=dev)
    flat_of_local[local[mine]] = x[mine]                            # this rank's local order -> flat index

    # reduce-to-owner: rank-order fp32 sum / world over the owned elements, written in place, + sum of squares
    grads = [torch.randn(n, generator=g, device=dev).to(torch.bfloat16) for _ in range(world)]
    want = (sum(t.float() for t in grads) * (1.0 / world)).to(torch.bfloat16)
    out = grads[rank]
    before = out.clone()
    part = torch.zeros(296, device=dev)
    sq = torch.zeros(1, device=dev)
    base = 0 if chunk else rank * seg
    C.reduce_owner(_ptrs(grads), out, base, seg, part, sq, chunk, rank)
    torch.cuda.synchronize()
    assert torch.equal(out[mine], want[mine]) and torch.equal(out[~mine], before[~mine])
    assert abs(sq.item() - want[mine].float().pow(2).sum().item()) <= 1e-3 * max(1.0, sq.item())

    # push all-gather: the owned elements land at the same flat index in every peer buffer, nothing else changes
    src = torch.randn(n, generator=g, device=dev).to(torch.bfloat16)
    peers = [torch.zeros(n, dtype=torch.bfloat16, device=dev) for _ in range(world)]
    peers[rank] = src
    C.push_range(src, _ptrs(peers), base, seg, rank, 64, chunk)
    torch.cuda.synchronize()
    for q in range(world):
        if q != rank:
            assert torch.equal(peers[q][mine], src[mine]) and not bool(peers[q][~mine].any())

    # Adam (and Adam fused with the push) reading / writing the bf16 buffers through the owner map
    hyper = torch.tensor([1e-3, 0.1, 0.001, 1.0], device=dev)
    factor = torch.tensor([0.5], device=dev)
    for fused in (False, True):
        p32 = torch.randn(seg, generator=g, device=dev)
        m = torch.rand(seg, generator=g, device=dev) * 0.1
        v = torch.rand(seg, generator=g, device=dev) * 0.1
        g16 = torch.randn(n, generator=g, device=dev).to(torch.bfloat16)
        p16 = torch.zeros(n, dtype=torch.bfloat16, device=dev)
        pr, mr, vr = p32.clone(), m.clone(), v.clone()
        gl = g16[flat_of_local]
        g_arg, p_arg = (g16, p16) if chunk else (g16[rank * seg:(rank + 1) * seg], p16[rank * seg:(rank + 1) * seg])
        if fused:
            pb = [torch.zeros(n, dtype=torch.bfloat16, device=dev) for _ in range(world)]
            pb[rank] = p16
            C.adam_push(p32, g_arg, m, v, p_arg, hyper, factor, 0.9, 0.95, 1e-8, 0.1, True, _ptrs(pb),
                        0 if chunk else rank * seg, rank, chunk)
        else:
            C.adam_step(p32, g_arg, m, v, p_arg, hyper, factor, 0.9, 0.95, 1e-8, 0.1, True, chunk, world, rank)
        torch.cuda.synchronize()
        # oracle with the same expression as the kernel (host-side bias corrections from the hyper vector)
        gg = gl.float() * 0.5
        mr = 0.9 * mr + 0.1 * gg
        vr = 0.95 * vr + 0.05 * gg * gg
        upd = (mr / 0.1) / ((vr / 0.001).sqrt() + 1e-8) + 0.1 * pr
        pr = pr - 1e-3 * upd
        assert torch.allclose(p32, pr, rtol=1e-5, atol=1e-6)
        assert torch.equal(p16[flat_of_local], p32.to(torch.bfloat16))
        assert not bool(p16[~mine].any())
        if fused:
            for q in range(world):
                if q != rank:
                    assert torch.equal(pb[q][mine], p16[mine]) and not bool(pb[q][~mine].any())

    # gradient push to the owners' staging slots (pieces cut at owner boundaries), then the staged owner sum
    stag = [torch.zeros(n, dtype=torch.bfloat16, device=dev) for _ in range(world)]
    arrive = [torch.zeros(64, dtype=torch.int32, device=dev) for _ in range(world)]
    gr = torch.randn(n, generator=g, device=dev).to(torch.bfloat16)
    step = chunk or seg
    pieces = [[o, min(step, n - o), int(owner[o])] for o in range(0, n, step) if int(owner[o]) != rank]
    C.push_grads(gr, _ptrs(stag), _ptrs(arrive), torch.tensor(pieces, dtype=torch.int64, device=dev), 0, rank, seg,
                 32, chunk)
    torch.cuda.synchronize()
    for q in range(world):
        if q == rank:
            assert not bool(stag[q].any())
            continue
        oq = owner == q
        slot = stag[q][rank * seg:(rank + 1) * seg]
        assert torch.equal(slot[local[oq]], gr[oq])
    # the owner's sum: its own values from its gradient buffer, every other rank r's from its staging slot r
    own_grad = torch.randn(n, generator=g, device=dev).to(torch.bfloat16)
    staging = torch.randn(n, generator=g, device=dev).to(torch.bfloat16)
    acc = torch.zeros(seg, device=dev)
    for r in range(world):
        acc += own_grad[flat_of_local].float() if r == rank else staging[r * seg:(r + 1) * seg].float()
    want = (acc * (1.0 / world)).to(torch.bfloat16)
    keep = own_grad.clone()
    C.reduce_compact(own_grad, staging, seg, world, rank, seg, chunk, part, 296)
    C.sum_partials(part, sq)
    torch.cuda.synchronize()
    assert torch.equal(own_grad[flat_of_local], want) and torch.equal(own_grad[~mine], keep[~mine])
    assert abs(sq.item() - want.float().pow(2).sum().item()) <= 1e-3 * max(1.0, sq.item())
    # the same sum over a table of owned pieces (flat offset, count), as the bucketed exchange runs it after the
    # copy engines delivered the other ranks' pieces
    own_grad = keep.clone()
    mine_pieces = [[o, min(step, n - o)] for o in range(0, n, step) if int(owner[o]) == rank]
    part.zero_()
    C.reduce_staged(own_grad, staging, torch.tensor(mine_pieces, dtype=torch.int64, device=dev), world, rank, seg,
                    part, 64, chunk)
    C.sum_partials(part, sq)
    torch.cuda.synchronize()
    assert torch.equal(own_grad[flat_of_local], want) and torch.equal(own_grad[~mine], keep[~mine])
    assert abs(sq.item() - want.float().pow(2).sum().item()) <= 1e-3 * max(1.0, sq.item())
    assert int(C.status()[0].item()) == 0


@pytest.mark.multigpu
def test_gemm_scatter_training_matches_serial_exchange(tmp_path):
    from faster_yoco_b200.utils import dist_checks
    from faster_yoco_b200.utils.launch import run_ranks
    run_ranks(dist_checks.gemm_scatter_vs_serial_gpu, 2, str(tmp_path), 4, backend="nccl", timeout_s=300)
    r = torch.load(os.path.join(tmp_path, "gemm_scatter.pt"))
    for name, base in (("gemm", "serial"), ("gemm_graph", "serial"), ("gemm_uf2", "serial_uf2"),
                       ("serial_cyclic", "serial"), ("gemm_cyclic", "serial"), ("gemm_cyclic_graph", "serial"),
                       ("gemm_overlap_cyclic", "serial"), ("sm_overlap_cyclic", "serial"),
                       ("pull_cyclic", "serial"), ("pull_cyclic_graph", "serial"), ("pull_even", "serial")):
        assert r[name]["status"] == 0 and r[base]["status"] == 0
        for a, b in zip(r[name]["losses"], r[base]["losses"]):
            assert abs(a - b) / abs(b) < 2e-4, (name, r[name]["losses"], r[base]["losses"])
        pf, ps = r[name]["params"], r[base]["params"]
        assert ((pf - ps).abs().max() / ps.abs().max()).item() < 1e-2, name


@pytest.mark.parametrize("chunk", [0, 1024])
def test_embedding_bwd_scatter_and_zero_staged(chunk):
    """The embedding's weight gradient with the touched rows stored at their owners (four ranks emulated in local
    memory) against the local embedding backward + the scatter oracle; then the owner clears the staging regions."""
    ops.set_backend("native")
    C = ops._C()
    dev = torch.device("cuda", 0)
    world, rank, V, N, M, x0 = 4, 3, 1000, 96, 700, 4096
    numel = V * N
    seg = int(math.ceil((x0 + numel) / (world * (chunk or 1024)))) * (chunk or 1024)
    g = torch.Generator(device=dev).manual_seed(11 + chunk)
    tok = torch.randint(0, V, (M,), generator=g, device=dev)
    dy = torch.randn(M, N, generator=g, device=dev).to(torch.bfloat16)
    grad_flat = torch.randn(world * seg, generator=g, device=dev).to(torch.bfloat16)
    staging = [torch.zeros(world * seg, dtype=torch.bfloat16, device=dev) for _ in range(world)]
    bases = torch.tensor([t.data_ptr() for t in staging], dtype=torch.int64, device=dev)
    want = C.embedding_bwd(tok, dy, V, 2.0, None)                  # dense [V, N], zero rows for unseen tokens
    own_exp = grad_flat.clone()
    own_exp[x0:x0 + numel] = 0
    stag_exp = [t.clone() for t in staging]
    # the oracle stores every row; the kernel only the touched ones, so the expected staging keeps zeros elsewhere
    ref.owner_scatter(want, x0, seg, rank, own_exp, stag_exp, chunk)
    slot = grad_flat[x0:x0 + numel].view(V, N)
    C.embedding_bwd_scatter(tok, dy, 2.0, slot, grad_flat, bases, seg, rank, chunk)
    torch.cuda.synchronize()
    assert torch.equal(grad_flat, own_exp)
    for q in range(world):
        assert torch.equal(staging[q], stag_exp[q]), q
    # an owner q clears, over its local ranges of this weight, every other rank's slot
    q = 1
    x = torch.arange(x0, x0 + numel, device=dev)
    o, loc = ref.zero_owner_local(x, seg, chunk, world)
    lq = loc[o == q]
    ranges = []
    lo = prev = None
    for v in lq.tolist():                                           # contiguous runs of local indices
        if lo is None:
            lo = prev = v
        elif v == prev + 1:
            prev = v
        else:
            ranges.append([lo, prev - lo + 1])
            lo = prev = v
    ranges.append([lo, prev - lo + 1])
    staging[q][q * seg:(q + 1) * seg] = 1.0                         # its own slot must stay untouched
    C.zero_staged(staging[q], torch.tensor(ranges, dtype=torch.int64, device=dev), world, q, seg, 16)
    torch.cuda.synchronize()
    for r in range(world):
        sl = staging[q][r * seg:(r + 1) * seg]
        if r == q:
            assert bool((sl == 1.0).all())
        else:
            assert not bool(sl[lq].any())
    assert int(C.status()[0].item()) == 0
