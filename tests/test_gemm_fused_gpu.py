"""Elementwise epilogues of the CTA-pair GEMM (gemm2.cu): the rotary embedding in the q / k projection, SwiGLU in
the merged fc1 | gate projection and the SwiGLU backward in the fc2 input gradient. Each is checked against the
separate kernels it replaces (same rounding points, so within one bf16 unit) and against an fp32 PyTorch oracle."""
import pytest
import torch

from faster_yoco_b200 import ops
from faster_yoco_b200.ops import reference as ref

pytestmark = pytest.mark.gpu


def C():
    return ops._C()


def dev():
    return torch.device("cuda", 0)


def rnd(*shape, seed, scale=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(*shape, device=dev(), generator=g) * scale).to(torch.bfloat16)


def close_ulps(x, y, ulps=1):
    """Elementwise |x - y| within `ulps` bf16 units of the larger magnitude (plus a tiny absolute floor)."""
    x, y = x.float(), y.float()
    mag = torch.maximum(x.abs(), y.abs()).clamp_min(1e-30)
    tol = ulps * torch.exp2(torch.floor(torch.log2(mag)) - 7) + 1e-6
    bad = (x - y).abs() > tol
    assert not bool(bad.any()), (int(bad.sum()), float((x - y).abs().max()))


def rel(x, r):
    if r.numel() == 0:
        return 0.0
    x, r = x.double(), r.double()
    return ((x - r).abs().max() / r.abs().max().clamp_min(1e-12)).item()


def tables(L, seed=0):
    ang = torch.rand(L, 64, device=dev(), generator=torch.Generator(device="cuda").manual_seed(seed)) * 6.283
    return ang.cos().to(torch.bfloat16).contiguous(), ang.sin().to(torch.bfloat16).contiguous()


@pytest.mark.parametrize("bn", [256, 192, 128])
@pytest.mark.parametrize("Bs,L,N,rot,K", [(2, 256, 1288, 512, 320), (1, 384, 3 * 256, 768, 256),
                                          (3, 128, 2 * 128 + 24, 256, 64)])
def test_gemm_rope_matches_gemm_then_rope(bn, Bs, L, N, rot, K):
    ops.set_backend("native")
    M = Bs * L
    a, w = rnd(M, K, seed=1, scale=0.5), rnd(N, K, seed=2, scale=0.5)
    cos, sin = tables(L + 7)
    y = torch.empty(M, N, dtype=torch.bfloat16, device=dev())
    C().gemm_rope(a, w, y, cos, sin, L, rot, bn)
    # separate kernels: the plain GEMM, then rope_fwd on the rotated head blocks
    y0 = ops.gemm(a, w)
    close_ulps(y[:, rot:], y0[:, rot:])
    q0 = C().rope_fwd(y0[:, :rot].view(Bs, L, rot // 128, 128), cos, sin, False)
    close_ulps(y[:, :rot].view(Bs, L, rot // 128, 128), q0)
    # fp32 oracle
    yf = a.float() @ w.float().t()
    qf = ref.apply_rope(yf[:, :rot].reshape(Bs, L, rot // 128, 128), cos[:L].float(), sin[:L].float())
    assert rel(y[:, :rot].reshape(Bs, L, rot // 128, 128), qf) < 1e-2
    assert rel(y[:, rot:], yf[:, rot:]) < 1e-2
    assert int(C().status()[0].item()) == 0


def test_gemm_rope_writes_strided_output():
    """The output may be a column block of a wider buffer (row stride > N)."""
    ops.set_backend("native")
    Bs, L, N, K = 2, 128, 512, 128
    a, w = rnd(Bs * L, K, seed=3), rnd(N, K, seed=4)
    cos, sin = tables(L)
    big = torch.zeros(Bs * L, N + 64, dtype=torch.bfloat16, device=dev())
    C().gemm_rope(a, w, big[:, 32:32 + N], cos, sin, L, 256, 256)
    y = torch.empty(Bs * L, N, dtype=torch.bfloat16, device=dev())
    C().gemm_rope(a, w, y, cos, sin, L, 256, 256)
    assert torch.equal(big[:, 32:32 + N], y)
    assert int(big[:, :32].abs().sum()) == 0 and int(big[:, 32 + N:].abs().sum()) == 0


@pytest.mark.parametrize("M,K,f", [(384, 320, 384), (256, 256, 160), (512, 192, 1024), (100, 128, 96)])
def test_gemm_swiglu_matches_gemm_then_swiglu(M, K, f):
    ops.set_backend("native")
    a, w = rnd(M, K, seed=5, scale=0.5), rnd(2 * f, K, seed=6, scale=0.5)
    u, h = C().gemm_swiglu(a, w)
    u0 = ops.gemm(a, w)
    close_ulps(u, u0)
    # h from the fused u equals the separate activation kernel on it
    close_ulps(h, C().swiglu_fwd(u[:, :f], u[:, f:]))
    uf = a.float() @ w.float().t()
    assert rel(u, uf) < 1e-2
    assert rel(h, ref.swiglu(uf[:, :f], uf[:, f:])) < 2e-2
    assert int(C().status()[0].item()) == 0


@pytest.mark.parametrize("M,K,f,pad", [(384, 320, 384, 0), (256, 128, 160, 64), (130, 256, 1024, 8)])
def test_gemm_swiglu_bwd_matches_gemm_then_swiglu_bwd(M, K, f, pad):
    ops.set_backend("native")
    g, w2 = rnd(M, K, seed=7, scale=0.5), rnd(K, f, seed=8, scale=0.5)
    ubig = rnd(M, 2 * f + pad, seed=9)
    u = ubig[:, :2 * f]                                   # row stride 2f + pad
    du = torch.empty(M, 2 * f, dtype=torch.bfloat16, device=dev())
    C().gemm_swiglu_bwd(g, w2, True, u, du)
    dh = ops.gemm(g, w2, b_mn_major=True)
    du0 = torch.empty_like(du)
    C().swiglu_bwd(u[:, :f], u[:, f:], dh, du0[:, :f], du0[:, f:])
    close_ulps(du, du0)
    # fp32 oracle
    dhf = g.float() @ w2.float()
    af, bf = u[:, :f].float(), u[:, f:].float()
    s = torch.sigmoid(af)
    assert rel(du[:, :f], s * (1 + af * (1 - s)) * dhf * bf) < 2e-2
    assert rel(du[:, f:], af * s * dhf) < 2e-2
    # K-major weight form ([f, K])
    du2 = torch.empty_like(du)
    C().gemm_swiglu_bwd(g, w2.t().contiguous(), False, u, du2)
    close_ulps(du2, du0)
    assert int(C().status()[0].item()) == 0


def _owner(x, seg, chunk, world):
    return (x // chunk) % world if chunk else x // seg


@pytest.mark.parametrize("world,chunk,bn,rope", [(4, 0, 256, False), (4, 4096, 256, False), (8, 2048, 192, True),
                                                 (2, 0, 192, False), (3, 8192, 256, True)])
def test_gemm_gather_pulls_owner_rows_and_multiplies(world, chunk, bn, rope):
    """The all-gather fused into the consumer GEMM, owners emulated by replicas in this GPU's memory: the weight's
    rows owned elsewhere are stale in this rank's replica before the call and current after it, the other elements
    of the replica are untouched, and the product uses the current rows."""
    ops.set_backend("native")
    K, N, L, Bs = 256, 648, 128, 3
    M = Bs * L
    span = (chunk or 1024) * world
    seg = ((N * K + 40960 + span - 1) // span) * span // world          # whole chunks / aligned segments
    rank = 1
    reps = [rnd(world * seg, seed=20 + r, scale=0.05) for r in range(world)]
    x = torch.arange(world * seg, device=dev())
    own = _owner(x, seg, chunk, world)
    truth = reps[0].clone()
    for r in range(world):
        truth[own == r] = reps[r][own == r]
    local = reps[rank]
    before = local.clone()
    peers = torch.tensor([t.data_ptr() for t in reps], dtype=torch.int64, device=dev())
    w_off = 8192 + 8 * 3                                          # 16-byte aligned, not tile aligned
    w = local[w_off:w_off + N * K].view(N, K)
    a = rnd(M, K, seed=30)
    y = torch.empty(M, N, dtype=torch.bfloat16, device=dev())
    if rope:
        cos, sin = tables(L)
        C().gemm_gather(a, w, y, local, peers, seg, chunk, rank, bn, cos, sin, L, 256)
    else:
        C().gemm_gather(a, w, y, local, peers, seg, chunk, rank, bn)
    torch.cuda.synchronize()
    assert int(C().status()[0].item()) == 0
    assert torch.equal(local[w_off:w_off + N * K], truth[w_off:w_off + N * K])
    assert torch.equal(local[:w_off], before[:w_off]) and torch.equal(local[w_off + N * K:], before[w_off + N * K:])
    wt = truth[w_off:w_off + N * K].view(N, K)
    if rope:
        y0 = torch.empty_like(y)
        C().gemm_rope(a, wt.contiguous(), y0, cos, sin, L, 256, bn)
    else:
        y0 = ops.gemm(a, wt.contiguous())
    close_ulps(y, y0)
