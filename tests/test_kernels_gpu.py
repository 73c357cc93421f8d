"""Numerics of every sm_100a kernel against a plain PyTorch fp32 reference of the same op."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def C():
    from faster_yoco_b200.ops import _native
    return _native.lib()


def rel(x, ref):
    x, ref = x.float(), ref.float()
    return ((x - ref).abs().max() / ref.abs().max().clamp_min(1e-6)).item()


def dev():
    return torch.device("cuda", 0)


# ------------------------------------------------------------------------------------------------------------------
# GEMM


GEMM_SHAPES = [(128, 256, 64), (256, 512, 192), (300, 520, 200), (2048, 3072, 3072), (512, 1000, 256),
               (2048, 12312, 3072), (130, 24, 72)]


@pytest.mark.parametrize("M,N,K", GEMM_SHAPES)
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True), (True, False)])
def test_gemm_majors(M, N, K, a_mn, b_mn):
    torch.manual_seed(M + N + K)
    a = torch.randn(M, K, device=dev(), dtype=torch.bfloat16)
    b = torch.randn(N, K, device=dev(), dtype=torch.bfloat16)
    ref = a.float() @ b.float().T
    A = a.T.contiguous() if a_mn else a
    B = b.T.contiguous() if b_mn else b
    if (a_mn and (M * 2) % 16) or (b_mn and (N * 2) % 16) or (K * 2) % 16:
        pytest.skip("TMA needs 16-byte row strides")
    out = torch.empty(M, N, device=dev(), dtype=torch.bfloat16)
    C().gemm(A, B, out, a_mn, b_mn, None)
    torch.cuda.synchronize()
    assert rel(out, ref) < 1e-2, (M, N, K, a_mn, b_mn, rel(out, ref))


def test_gemm_residual_and_f32():
    M, N, K = 640, 768, 512
    a = torch.randn(M, K, device=dev(), dtype=torch.bfloat16)
    b = torch.randn(N, K, device=dev(), dtype=torch.bfloat16)
    r = torch.randn(M, N, device=dev(), dtype=torch.bfloat16)
    ref = a.float() @ b.float().T
    out = torch.empty(M, N, device=dev(), dtype=torch.bfloat16)
    C().gemm(a, b, out, False, False, r)
    exp = (ref.to(torch.bfloat16).float() + r.float())
    assert rel(out, exp) < 1e-2
    o32 = torch.empty(M, N, device=dev(), dtype=torch.float32)
    C().gemm(a, b, o32, False, False, None)
    assert rel(o32, ref) < 1e-4
    # in-place accumulate: out = a b^T + out
    acc = r.clone()
    C().gemm(a, b, acc, False, False, acc)
    assert rel(acc, exp) < 1e-2
    assert int(C().status()[0].item()) == 0


def test_gemm_linear_autograd():
    from faster_yoco_b200 import ops
    ops.set_backend("native")
    x = torch.randn(2, 256, 512, device=dev(), dtype=torch.bfloat16, requires_grad=True)
    w = torch.randn(384, 512, device=dev(), dtype=torch.bfloat16, requires_grad=True) * 0.05
    w = w.detach().requires_grad_()
    y = ops.linear(x, w)
    g = torch.randn_like(y)
    y.backward(g)
    xf, wf = x.detach().float().requires_grad_(), w.detach().float().requires_grad_()
    yf = xf @ wf.T
    yf.backward(g.float())
    assert rel(y, yf) < 1e-2
    assert rel(x.grad, xf.grad) < 1e-2
    assert rel(w.grad, wf.grad) < 1e-2


# ------------------------------------------------------------------------------------------------------------------
# norms / elementwise


@pytest.mark.parametrize("M,N", [(2048, 3072), (37, 256), (5, 688)])
def test_rms_norm(M, N):
    from faster_yoco_b200.ops import reference as ref
    x = torch.randn(M, N, device=dev(), dtype=torch.bfloat16) * 3
    w = (torch.rand(N, device=dev()) + 0.5).to(torch.bfloat16)
    y, rstd = C().rms_norm_fwd(x, w, 1e-5)
    assert rel(y, ref.rms_norm(x, w, 1e-5)) < 1e-2
    dy = torch.randn_like(x)
    dx, dw = C().rms_norm_bwd(dy, x, w, rstd)
    xf, wf = x.float().requires_grad_(), w.float().requires_grad_()
    yf = ref.rms_norm(xf, wf, 1e-5)
    yf.backward(dy.float())
    assert rel(dx, xf.grad) < 2e-2
    assert rel(dw, wf.grad) < 2e-2


def test_swiglu():
    from faster_yoco_b200.ops import reference as ref
    h = torch.randn(300, 2 * 688, device=dev(), dtype=torch.bfloat16) * 2
    x, y = h[:, :688], h[:, 688:]
    out = C().swiglu_fwd(x, y)
    assert rel(out, ref.swiglu(x, y)) < 1e-2
    g = torch.randn(300, 688, device=dev(), dtype=torch.bfloat16)
    dx, dy = C().swiglu_bwd(x, y, g)
    xf, yf = x.float().requires_grad_(), y.float().requires_grad_()
    (xf * yf * torch.sigmoid(xf)).backward(g.float())
    assert rel(dx, xf.grad) < 2e-2 and rel(dy, yf.grad) < 2e-2


def test_rope_strided_and_conj():
    from faster_yoco_b200.ops import reference as ref
    B, L, H, D = 2, 300, 3, 128
    big = torch.randn(B, L, 5 * H * D, device=dev(), dtype=torch.bfloat16)
    x = big[..., H * D:2 * H * D].view(B, L, H, D)
    cos, sin = ref.rope_tables(D, 0, L, 1e4, torch.bfloat16, dev())
    out = C().rope_fwd(x, cos, sin, False)
    assert rel(out, ref.apply_rope(x, cos, sin)) < 1e-2
    back = C().rope_fwd(out, cos, sin, True)
    assert rel(back, x) < 2e-2


@pytest.mark.parametrize("D", [128, 64])
def test_rope_neox(D):
    from faster_yoco_b200.ops import reference as ref
    B, L, H = 2, 77, 4
    big = torch.randn(B, L, 3 * H * D, device=dev(), dtype=torch.bfloat16)
    x = big[..., H * D:2 * H * D].view(B, L, H, D)
    ang = ref.llama_rope_angles(D, L, 1e4, dev())
    cos, sin = torch.cos(ang).to(torch.bfloat16), torch.sin(ang).to(torch.bfloat16)
    out = C().rope_fwd(x, cos, sin, False, True)
    assert rel(out, ref.apply_rope(x, cos, sin, interleaved=False)) < 1e-2
    back = C().rope_fwd(out, cos, sin, True, True)
    assert rel(back, x) < 2e-2


def test_subln_swiglu():
    from faster_yoco_b200.ops import reference as ref
    T, H, D = 257, 6, 128
    o = torch.randn(T, H * D, device=dev(), dtype=torch.bfloat16)
    big = torch.randn(T, 5 * H * D, device=dev(), dtype=torch.bfloat16)
    g = big[:, 3 * H * D:4 * H * D]
    out, rstd = C().subln_swiglu_fwd(o, g, 1e-5, D)
    on = ref.rms_norm(o.view(T, H, D), None, 1e-5).view(T, H * D)
    assert rel(out, ref.swiglu(g, on)) < 1e-2
    dout = torch.randn_like(out)
    do, dg = C().subln_swiglu_bwd(dout, o, g, rstd, D)
    of, gf = o.float().requires_grad_(), g.float().requires_grad_()
    onf = ref.rms_norm(of.view(T, H, D), None, 1e-5).view(T, H * D)
    (gf * onf * torch.sigmoid(gf)).backward(dout.float())
    assert rel(do, of.grad) < 3e-2 and rel(dg, gf.grad) < 2e-2


@pytest.mark.parametrize("M", [513, 20000])
def test_embedding(M):
    V, N = 1000, 256
    w = torch.randn(V, N, device=dev(), dtype=torch.bfloat16)
    tok = torch.randint(0, V, (M,), device=dev())
    tok[:20] = 7                       # repeated tokens
    scale = math.sqrt(N)
    out = C().embedding_fwd(tok, w, scale)
    assert rel(out, w[tok].float() * scale) < 1e-2
    dy = torch.randn(M, N, device=dev(), dtype=torch.bfloat16)
    dw = C().embedding_bwd(tok, dy, V, scale, None)
    ref = torch.zeros(V, N, device=dev()).index_add_(0, tok, dy.float() * scale)
    assert rel(dw, ref) < 2e-2


@pytest.mark.parametrize("V", [100288, 1024, 1003])
def test_cross_entropy(V):
    from faster_yoco_b200.ops import reference as ref
    M = 64
    x = (torch.randn(M, V, device=dev()) * 3).to(torch.bfloat16)
    t = torch.randint(0, V, (M,), device=dev())
    t[:5] = 1                          # padding targets
    loss, lse = C().ce_fwd(x, t, 1)
    r = ref.cross_entropy_sum(x, t, 1)
    assert abs(loss.sum().item() - r.item()) / abs(r.item()) < 1e-4
    g = torch.tensor([0.37], device=dev())
    dx = C().ce_bwd(x, t, lse, g, 1, None)
    xf = x.float().requires_grad_()
    (ref.cross_entropy_sum(xf, t, 1) * 0.37).backward()
    assert rel(dx, xf.grad) < 1e-2


def test_adam_matches_reference_and_sq_norm():
    from faster_yoco_b200.ops import reference as ref
    n = 100003
    p = torch.randn(n, device=dev())
    m = torch.randn(n, device=dev()).abs() * 1e-3
    v = torch.rand(n, device=dev()) * 1e-6
    g16 = (torch.randn(n, device=dev()) * 1e-2).to(torch.bfloat16)
    p16 = torch.empty(n, device=dev(), dtype=torch.bfloat16)
    lr, b1, b2, eps, wd, step, factor = 1.5e-4, 0.9, 0.95, 1e-6, 0.05, 7, 0.75
    bc1 = float(torch.tensor(1 - b1 ** step, dtype=torch.float32))
    bc2 = float(torch.tensor(1 - b2 ** step, dtype=torch.float32))
    hyper = torch.tensor([lr, bc1, bc2, step], device=dev(), dtype=torch.float32)
    fac = torch.tensor([factor], device=dev())
    p_r, m_r, v_r = p.clone(), m.clone(), v.clone()
    C().adam_step(p, g16, m, v, p16, hyper, fac, b1, b2, eps, wd, True)
    ref.adam_step_(p_r, g16.float() * factor, m_r, v_r, lr=lr, beta1=b1, beta2=b2, eps=eps, step=step,
                   weight_decay=wd, adamw=True)
    assert (p - p_r).abs().max().item() < 1e-6
    assert (m - m_r).abs().max().item() < 1e-9
    assert torch.equal(p16, p.to(torch.bfloat16))
    x = torch.randn(3_000_001, device=dev()).to(torch.bfloat16)
    s = C().sq_norm(x)
    r = x.double().pow(2).sum()
    assert abs(s.item() - r.item()) / r.item() < 1e-4


@pytest.mark.parametrize("M,N,K", [(2048, 3072, 16384), (2048, 3072, 100288)])
def test_gemm_split_k_with_residual(M, N, K):
    """Long-K / small-output shapes take the split-K path (fp32 slice partials + ordered reduction)."""
    torch.manual_seed(7)
    a = torch.randn(M, K, device=dev(), dtype=torch.bfloat16)
    b = torch.randn(N, K, device=dev(), dtype=torch.bfloat16) * 0.05
    r = torch.randn(M, N, device=dev(), dtype=torch.bfloat16)
    ref = a.float() @ b.float().T
    out = torch.empty(M, N, device=dev(), dtype=torch.bfloat16)
    C().gemm(a, b.T.contiguous(), out, False, True, r)     # dgrad layout: B MN-major
    assert rel(out, ref.to(torch.bfloat16).float() + r.float()) < 1e-2
    out2 = torch.empty(M, N, device=dev(), dtype=torch.bfloat16)
    C().gemm(a, b, out2, False, False, None)
    assert rel(out2, ref) < 1e-2


def test_sq_norm_ranges_any_alignment():
    """Sum of squares over many ranges of one bf16 buffer (unaligned starts, lengths up to 65,536) in one launch,
    against fp64 PyTorch; the order of the partials is fixed, so two calls agree bit for bit."""
    lib = C()
    dv = dev()
    g = torch.Generator(device=dv).manual_seed(3)
    x = torch.randn(1 << 20, generator=g, device=dv).to(torch.bfloat16)
    rows = [[0, 65536], [3, 17], [70001, 65536], [200003, 1], [300000, 40000], [1048575, 1], [500001, 9]]
    chunks = torch.tensor(rows, dtype=torch.int64, device=dv)
    got = lib.sq_norm_ranges(x, chunks)
    want = sum(x[a:a + n].double().pow(2).sum().item() for a, n in rows)
    assert abs(got.item() - want) <= 1e-5 * want
    assert torch.equal(got, lib.sq_norm_ranges(x, chunks))
    empty = lib.sq_norm_ranges(x, torch.zeros(0, 2, dtype=torch.int64, device=dv))
    assert empty.item() == 0.0
