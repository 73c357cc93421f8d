"""tcgen05 attention / retention kernels vs plain PyTorch fp32 references (forward and backward)."""
import pytest
import torch

from faster_yoco_b200 import ops
from faster_yoco_b200.ops import reference as ref

pytestmark = pytest.mark.gpu


def rel(x, r):
    x, r = x.float(), r.float()
    return ((x - r).abs().max() / r.abs().max().clamp_min(1e-6)).item()


def dev():
    return torch.device("cuda", 0)


def strided_heads(B, L, H, D, extra=3, seed=0):
    """[B, L, H, D] view with a token stride larger than H*D (like a column block of a fused projection)."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    big = torch.randn(B, L, (H + extra) * D, device=dev(), dtype=torch.float32, generator=g).to(torch.bfloat16)
    return big[..., D:(H + 1) * D].view(B, L, H, D)


@pytest.mark.parametrize("B,L,Hq,Hk,window", [(1, 256, 2, 2, None), (2, 300, 6, 2, None), (1, 2048, 3, 1, None),
                                              (1, 1000, 4, 4, 200), (1, 130, 2, 1, None)])
def test_attention_fwd_bwd(B, L, Hq, Hk, window):
    ops.set_backend("native")
    D = 128
    q = strided_heads(B, L, Hq, D, seed=1).requires_grad_()
    k = strided_heads(B, L, Hk, D, seed=2).requires_grad_()
    v = strided_heads(B, L, Hk, D, seed=3).requires_grad_()
    o = ops.attention(q, k, v, causal=True, window=window)
    do = torch.randn_like(o)
    o.backward(do)
    qf, kf, vf = (t.detach().float().requires_grad_() for t in (q, k, v))
    of = ref.attention(qf, kf, vf, causal=True, window=window)
    of.backward(do.float())
    assert rel(o, of) < 2e-2
    assert rel(q.grad, qf.grad) < 3e-2
    assert rel(k.grad, kf.grad) < 3e-2
    assert rel(v.grad, vf.grad) < 3e-2
    assert int(ops._C().status()[0].item()) == 0


@pytest.mark.parametrize("form", ["chunk", "parallel"])
@pytest.mark.parametrize("B,L,H", [(1, 256, 2), (2, 384, 3), (1, 2048, 2), (1, 200, 1)])
def test_retention_fwd_bwd(B, L, H, form, monkeypatch):
    """Both native forms: the chunkwise kernels (default) and the quadratic parallel-form kernel."""
    ops.set_backend("native")
    monkeypatch.setattr(ops, "RETENTION_FORM", form)
    D = 128
    q = strided_heads(B, L, H, D, seed=4).requires_grad_()
    k = strided_heads(B, L, H, D, seed=5).requires_grad_()
    v = strided_heads(B, L, H, D, seed=6).requires_grad_()
    graw = torch.randn(B, L, H, device=dev(), requires_grad=True)
    gt = torch.nn.functional.logsigmoid(graw) / 16
    o = ops.retention(q, k, v, gt)
    do = torch.randn_like(o)
    o.backward(do)
    qf, kf, vf = (t.detach().float().requires_grad_() for t in (q, k, v))
    grf = graw.detach().clone().requires_grad_()
    gtf = torch.nn.functional.logsigmoid(grf) / 16
    of = ref.parallel_gate_retention_f32(qf.transpose(1, 2), kf.transpose(1, 2), vf.transpose(1, 2),
                                         gtf.transpose(1, 2)).transpose(1, 2)
    of.backward(do.float())
    assert rel(o, of) < 2e-2
    assert rel(q.grad, qf.grad) < 3e-2
    assert rel(k.grad, kf.grad) < 3e-2
    assert rel(v.grad, vf.grad) < 3e-2
    assert rel(graw.grad, grf.grad) < 5e-2
    assert int(ops._C().status()[0].item()) == 0
