"""Chunkwise gated-retention kernels (retention.cu) against PyTorch references in fp64 / fp32: forward and backward
at short, training and long sequence lengths, ordinary and strongly negative gates, entering / leaving states, the
chunked prefill (with and without a padding mask) and the decode step."""
import math

import pytest
import torch
import torch.nn.functional as F

from faster_yoco_b200 import ops
from faster_yoco_b200.ops import reference as ref

pytestmark = pytest.mark.gpu

D = 128


def rel(x, r):
    x, r = x.double(), r.double()
    return ((x - r).abs().max() / r.abs().max().clamp_min(1e-12)).item()


def dev():
    return torch.device("cuda", 0)


def heads(B, L, H, seed, extra=2):
    """[B, L, H, 128] bf16 view with a token stride wider than H * 128 (like a block of a fused projection)."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    big = torch.randn(B, L, (H + extra) * D, device=dev(), generator=g).to(torch.bfloat16)
    return big[..., D:(H + 1) * D].view(B, L, H, D)


def gates(B, L, H, seed, strong=False):
    g = torch.Generator(device="cuda").manual_seed(seed)
    raw = torch.randn(B, L, H, device=dev(), generator=g)
    if strong:
        raw = raw - 20.0                     # log-sigmoid ~ -20, /16: ~ -1.25 per step (tiles underflow)
    return raw


def oracle(q, k, v, g, state=None):
    """o [B, L, H, D] and the leaving state in fp64: the recurrence run chunk by chunk (exact, any L).
    q, k, v: [B, L, H, D]; g: [B, L, H] per-step log decays; state: [B, H, D, D] or None."""
    B, L, H, _ = q.shape
    qd, kd, vd = (t.double().transpose(1, 2) for t in (q, k, v))
    kd = kd / math.sqrt(D)
    gd = g.double().transpose(1, 2)
    S = torch.zeros(B, H, D, D, dtype=torch.float64, device=q.device) if state is None else state.double().clone()
    out = []
    C = 256
    for c0 in range(0, L, C):
        c1 = min(L, c0 + C)
        gl = gd[..., c0:c1].cumsum(-1)                              # [B, H, n]
        qc, kc, vc = qd[:, :, c0:c1], kd[:, :, c0:c1], vd[:, :, c0:c1]
        n = c1 - c0
        E = (gl[..., :, None] - gl[..., None, :])
        mask = torch.ones(n, n, dtype=torch.bool, device=q.device).tril()
        E = torch.where(mask, E.clamp(max=0).exp(), torch.zeros((), dtype=torch.float64, device=q.device))
        o = (qc @ kc.transpose(-1, -2) * E) @ vc + (qc * gl[..., None].exp()) @ S
        out.append(o)
        tot = gl[..., -1:]
        S = S * tot[..., None].exp() + kc.transpose(-1, -2) @ (vc * (tot - gl).exp()[..., None])
    return torch.cat(out, 2).transpose(1, 2), S


@pytest.mark.parametrize("B,L,H,strong", [(1, 200, 2, False), (2, 384, 3, False), (1, 2048, 2, False),
                                          (1, 2048, 2, True), (2, 300, 2, True), (1, 130, 1, False)])
def test_chunk_retention_fwd_bwd_vs_fp64(B, L, H, strong):
    ops.set_backend("native")
    q = heads(B, L, H, 1).requires_grad_()
    k = heads(B, L, H, 2).requires_grad_()
    v = heads(B, L, H, 3).requires_grad_()
    graw = gates(B, L, H, 4, strong).requires_grad_()
    o = ops.retention(q, k, v, F.logsigmoid(graw) / 16)
    do = torch.randn_like(o)
    o.backward(do)
    qf, kf, vf = (t.detach().double().requires_grad_() for t in (q, k, v))
    gf = graw.detach().double().requires_grad_()
    of, _ = oracle(qf, kf, vf, F.logsigmoid(gf) / 16)
    of.backward(do.double())
    assert rel(o, of) < 2e-2
    assert rel(q.grad, qf.grad) < 3e-2
    assert rel(k.grad, kf.grad) < 3e-2
    assert rel(v.grad, vf.grad) < 3e-2
    assert rel(graw.grad, gf.grad) < 5e-2
    assert int(ops._C().status()[0].item()) == 0


def test_chunk_retention_long_sequence_fwd():
    """L = 16,384: the chunk-local cumsum keeps the decay exponents exact however far apart the positions are."""
    ops.set_backend("native")
    B, L, H = 1, 16384, 2
    q, k, v = heads(B, L, H, 5), heads(B, L, H, 6), heads(B, L, H, 7)
    for strong in (False, True):
        g = F.logsigmoid(gates(B, L, H, 8, strong)) / 16
        o = ops.retention(q, k, v, g)
        of, _ = oracle(q, k, v, g)
        assert rel(o, of) < 2e-2, strong
    assert int(ops._C().status()[0].item()) == 0


def test_chunk_retention_long_sequence_bwd():
    ops.set_backend("native")
    B, L, H = 1, 16384, 1
    q = heads(B, L, H, 9).requires_grad_()
    k = heads(B, L, H, 10).requires_grad_()
    v = heads(B, L, H, 11).requires_grad_()
    graw = gates(B, L, H, 12).requires_grad_()
    o = ops.retention(q, k, v, F.logsigmoid(graw) / 16)
    do = torch.randn_like(o)
    o.backward(do)
    qf, kf, vf = (t.detach().double().requires_grad_() for t in (q, k, v))
    gf = graw.detach().double().requires_grad_()
    of, _ = oracle(qf, kf, vf, F.logsigmoid(gf) / 16)
    of.backward(do.double())
    for a, b in ((q.grad, qf.grad), (k.grad, kf.grad), (v.grad, vf.grad)):
        assert rel(a, b) < 3e-2
    assert rel(graw.grad, gf.grad) < 5e-2


@pytest.mark.parametrize("L", [256, 200])
def test_chunk_retention_states_in_and_out(L):
    """Entering state in, leaving state out, gradients of both (the context-parallel / prefill interface)."""
    ops.set_backend("native")
    C = ops._C()
    B, H = 2, 2
    q, k, v = heads(B, L, H, 13), heads(B, L, H, 14), heads(B, L, H, 15)
    g = (F.logsigmoid(gates(B, L, H, 16)) / 16).transpose(1, 2).contiguous()       # [B, H, L]
    s_in = torch.randn(B, H, D, D, device=dev()) * 0.1
    gloc = C.retention_chunk_cumsum(g)
    o, states, s_out = C.retention_chunk_fwd(q, k, v, gloc, state_in=s_in, want_state=True)
    of, sf = oracle(q, k, v, g.transpose(1, 2), s_in)
    assert rel(o, of) < 2e-2
    assert rel(s_out, sf) < 1e-2
    # state only (no outputs) agrees with the full forward
    assert rel(C.retention_chunk_state(k, v, gloc, state_in=s_in), sf) < 1e-2
    # backward with both state gradients against fp64 autograd
    do = torch.randn(B, L, H, D, device=dev()).to(torch.bfloat16)
    ds_out = torch.randn(B, H, D, D, device=dev()) * 0.1
    dq, dk, dv, ds_in, _ = C.retention_chunk_bwd(do, q, k, v, gloc, states, dstate_out=ds_out, want_dstate_in=True,
                                                 has_state_in=True)
    qf, kf, vf = (t.double().requires_grad_() for t in (q, k, v))
    sfi = s_in.double().requires_grad_()
    of2, sf2 = oracle(qf, kf, vf, g.transpose(1, 2), sfi)
    (of2 * do.double()).sum().add_((sf2 * ds_out.double()).sum()).backward()
    assert rel(dq, qf.grad) < 3e-2
    assert rel(dk, kf.grad) < 3e-2
    assert rel(dv, vf.grad) < 3e-2
    assert rel(ds_in, sfi.grad) < 2e-2
    assert int(C.status()[0].item()) == 0


def test_prefill_blocks_then_decode_match_one_pass():
    """Prefill in two blocks (state carried), then decode steps, equals one pass over the whole sequence."""
    ops.set_backend("native")
    B, H, L1, L2, n_dec = 2, 3, 256, 200, 4
    L = L1 + L2 + n_dec
    q, k, v = heads(B, L, H, 17), heads(B, L, H, 18), heads(B, L, H, 19)
    g = F.logsigmoid(gates(B, L, H, 20)) / 16
    of, sf = oracle(q, k, v, g)
    blk = lambda t, a, b: t[:, a:b].contiguous()       # the kernels take one token stride for the whole batch
    o1, s = ops.retention_prefill(blk(q, 0, L1), blk(k, 0, L1), blk(v, 0, L1), g[:, :L1])
    o2, s = ops.retention_prefill(blk(q, L1, L1 + L2), blk(k, L1, L1 + L2), blk(v, L1, L1 + L2), g[:, L1:L1 + L2], s)
    outs = [o1, o2]
    for t in range(L1 + L2, L):
        outs.append(ops.retention_decode(q[:, t:t + 1].contiguous(), k[:, t:t + 1].contiguous(),
                                         v[:, t:t + 1].contiguous(), g[:, t:t + 1], s))
    o = torch.cat(outs, 1)
    assert rel(o, of) < 2e-2
    assert rel(s, sf) < 1e-2


def test_decode_step_matches_reference_recurrence():
    ops.set_backend("native")
    B, H = 3, 4
    q, k, v = heads(B, 1, H, 21), heads(B, 1, H, 22), heads(B, 1, H, 23)
    g = F.logsigmoid(gates(B, 1, H, 24)) / 16
    state = torch.randn(B, H, D, D, device=dev())
    o_ref, s_ref = ref.recurrent_gate_retention(q.float().transpose(1, 2), k.float().transpose(1, 2),
                                                v.float().transpose(1, 2), g.transpose(1, 2), state.clone())
    s = state.clone()
    o = ops.retention_decode(q.contiguous(), k.contiguous(), v.contiguous(), g, s)
    assert rel(o[:, 0], o_ref[:, :, 0]) < 1e-2
    assert rel(s, s_ref) < 1e-5


def test_prefill_padding_mask_matches_reference():
    """A padded prefill block: outputs use every position, the state skips the padded ones (reference semantics)."""
    ops.set_backend("native")
    B, H, L, pad = 2, 2, 256, 40
    q, k, v = heads(B, L, H, 25), heads(B, L, H, 26), heads(B, L, H, 27)
    g = F.logsigmoid(gates(B, L, H, 28)) / 16
    mask = torch.arange(L, device=dev()) >= L - pad
    last = torch.randn(B, H, D, D, device=dev()) * 0.1
    o, s = ops.retention_prefill(q, k, v, g, last, mask)
    qh, kh, vh, gh = (t.float().transpose(1, 2) for t in (q, k, v, g))
    s_ref = ref.retention_prefill_state(kh, vh, gh, mask, last)
    of, _ = oracle(q, k, v, g, last)
    assert rel(o, of) < 2e-2
    assert rel(s, s_ref) < 1e-2
