"""Whole decoder layers as single autograd Functions for the native training path.

The module code in :mod:`faster_yoco_b200.models.layers` expresses a layer as a chain of ops, and autograd then
pays for the glue between them: a zero-filled gradient per slice of every fused projection output, a bf16 add per
residual branch, a ``.contiguous()`` copy per strided gradient. Here each layer's backward is written out:

* the residual gradient is added inside the RMSNorm backward kernel (``dres``),
* the mixer writes its gradients straight into column blocks of the fused projection's gradient (retention: dq / dk
  leave the kernels through the conjugate rotation, dv and dg are written in place, the gate gradient comes from
  the reverse-cumsum kernel),
* weight gradients go to the flat ZeRO gradient buffer (``ops._grad_slot``),

so a layer's backward is its GEMMs plus one kernel per op. Same math as the module path (which remains the CPU and
inference path); used when training on CUDA with head_dim 128 and no incremental state.
"""
from __future__ import annotations

from typing import Tuple

import torch

from .. import ops


def _C():
    return ops._C()


def _wgrad(w: torch.Tensor, dy: torch.Tensor, x: torch.Tensor):
    """dW = dy^T x into w's gradient slot or at its ZeRO owners (returns None), or as a new tensor."""
    if ops.wgrad_into(w, dy, x):
        return None
    return ops.gemm(dy, x, a_mn_major=True, b_mn_major=True)


def _ngrad(w: torch.Tensor, dw: torch.Tensor):
    slot, acc = ops._grad_slot(w)
    if slot is not None:
        slot.add_(dw) if acc else slot.copy_(dw)
        return None
    return dw


def _fuse_ok(f: int) -> bool:
    """The fused GEMM epilogues apply (FYB_GEMM_FUSE on, widths the 16-byte stores and 32-column chunks cover)."""
    return ops.GEMM_FUSE and f % 32 == 0


def _ffn_forward(x1, wn2, wfc1g, wfc2, eps, f):
    C = _C()
    h2, r2 = C.rms_norm_fwd(x1, wn2, eps)
    if _fuse_ok(f):
        u, a = ops.gemm_swiglu(h2, wfc1g)          # SwiGLU in the fc1 | gate GEMM's epilogue
    else:
        u = ops.gemm(h2, wfc1g)
        a = C.swiglu_fwd(u[:, :f], u[:, f:])
    xo = ops.gemm(a, wfc2, residual=x1)
    return xo, (h2, r2, u, a)


def _ffn_backward(dxo, x1, wn2, wfc1g, wfc2, saved, f):
    """Returns (dx1 including the residual gradient, grads for wn2, wfc1g, wfc2)."""
    C = _C()
    h2, r2, u, a = saved
    T = dxo.shape[0]
    du = torch.empty(T, 2 * f, dtype=dxo.dtype, device=dxo.device)
    if _fuse_ok(f):
        ops.gemm_swiglu_bwd(dxo, wfc2, u, du)       # the SwiGLU backward in the fc2 input-gradient epilogue
    else:
        da = ops.gemm(dxo, wfc2, b_mn_major=True)
        C.swiglu_bwd(u[:, :f], u[:, f:], da, du[:, :f], du[:, f:])
    g_fc2 = _wgrad(wfc2, dxo, a)
    dh2 = ops.gemm(du, wfc1g, b_mn_major=True)
    g_fc1g = _wgrad(wfc1g, du, h2)
    dx1, dwn2 = C.rms_norm_bwd(dh2, x1, wn2, r2, dxo)
    return dx1, _ngrad(wn2, dwn2), g_fc1g, g_fc2


class SelfRetentionLayerFn(torch.autograd.Function):
    """x -> x + out(swiglu(g, subln(retention(rope q, rope k, v, gates)))) -> + fc2(swiglu(fc1, gate))."""

    @staticmethod
    def forward(ctx, x, wn1, wqkvg, wout, wn2, wfc1g, wfc2, cos, sin, cfg):
        C = _C()
        H, D, eps, sub_eps, norm, f = cfg
        B, L, d = x.shape
        T = B * L
        R = wqkvg.shape[0]
        x2 = x.reshape(T, d)
        h1, r1 = C.rms_norm_fwd(x2, wn1, eps)
        if _fuse_ok(d):
            # q, k rotated in the projection's epilogue, read in place from y
            y = ops.gemm_rope(h1, wqkvg, cos, sin, L, 2 * d)
            y3 = y.view(B, L, R)
            q = y3[..., :d].view(B, L, H, D)
            k = y3[..., d:2 * d].view(B, L, H, D)
        else:
            y = ops.gemm(h1, wqkvg)
            y3 = y.view(B, L, R)
            q = C.rope_fwd(y3[..., :d].view(B, L, H, D), cos, sin, False)
            k = C.rope_fwd(y3[..., d:2 * d].view(B, L, H, D), cos, sin, False)
        v = y3[..., 2 * d:3 * d].view(B, L, H, D)
        if ops.RETENTION_FORM == "parallel":
            gcum = C.gate_cumsum_fwd(y[:, 4 * d:4 * d + H], B, L, float(norm))
            o = C.retention_fwd(q, k, v, gcum)
            states = gcum
        else:                      # chunkwise: chunk-local gate cumsum, entering states kept for the backward
            gcum = C.gate_cumsum_fwd(y[:, 4 * d:4 * d + H], B, L, float(norm), True)
            o, states, _ = C.retention_chunk_fwd(q, k, v, gcum)
        o2, rs = C.subln_swiglu_fwd(o.view(T, d), y[:, 3 * d:4 * d], float(sub_eps), D)
        x1 = ops.gemm(o2, wout, residual=x2)
        xo, ffn_saved = _ffn_forward(x1, wn2, wfc1g, wfc2, eps, f)
        ctx.save_for_backward(x2, h1, r1, y, q, k, gcum, o, rs, o2, x1, *ffn_saved, wn1, wqkvg, wout, wn2, wfc1g,
                              wfc2, cos, sin, states)
        ctx.cfg = cfg
        ctx.shape = (B, L, d)
        return xo.view(B, L, d)

    @staticmethod
    def backward(ctx, dxo):
        C = _C()
        (x2, h1, r1, y, q, k, gcum, o, rs, o2, x1, h2, r2, u, a, wn1, wqkvg, wout, wn2, wfc1g, wfc2, cos,
         sin, states) = ctx.saved_tensors
        H, D, eps, sub_eps, norm, f = ctx.cfg
        B, L, d = ctx.shape
        T = B * L
        R = wqkvg.shape[0]
        dxo = dxo.reshape(T, d).contiguous()
        dx1, g_n2, g_fc1g, g_fc2 = _ffn_backward(dxo, x1, wn2, wfc1g, wfc2, (h2, r2, u, a), f)
        do2 = ops.gemm(dx1, wout, b_mn_major=True)
        g_out = _wgrad(wout, dx1, o2)
        dy = torch.empty(T, R, dtype=dxo.dtype, device=dxo.device)
        dy3 = dy.view(B, L, R)
        do, _ = C.subln_swiglu_bwd(do2, o.view(T, d), y[:, 3 * d:4 * d], rs, D, dy[:, 3 * d:4 * d])
        v = y.view(B, L, R)[..., 2 * d:3 * d].view(B, L, H, D)
        dqv, dkv, dvv = (dy3[..., i * d:(i + 1) * d].view(B, L, H, D) for i in range(3))
        if ops.RETENTION_FORM == "parallel":
            _, _, _, dg = C.retention_bwd(do.view(B, L, H, D), q, k, v, gcum, o, dqv, dkv, dvv, cos, sin)
        else:
            dg = C.retention_chunk_bwd(do.view(B, L, H, D), q, k, v, gcum, states, dq=dqv, dk=dkv, dv=dvv,
                                       rope_cos=cos, rope_sin=sin, want_dgate=True)[4]
        ydg = dy[:, 4 * d:4 * d + H]
        C.gate_cumsum_bwd(dg, y[:, 4 * d:4 * d + H], ydg, float(norm))
        if R > 4 * d + H:
            dy[:, 4 * d + H:].zero_()
        dh1 = ops.gemm(dy, wqkvg, b_mn_major=True)
        g_qkvg = _wgrad(wqkvg, dy, h1)
        dx, dwn1 = C.rms_norm_bwd(dh1, x2, wn1, r1, dx1)
        return (dx.view(B, L, d), _ngrad(wn1, dwn1), g_qkvg, g_out, g_n2, g_fc1g, g_fc2, None, None, None)


class SelfWindowLayerFn(torch.autograd.Function):
    """Sliding-window attention self layer: q, k rotated, causal softmax attention over the last `window` keys."""

    @staticmethod
    def forward(ctx, x, wn1, wqkv, wout, wn2, wfc1g, wfc2, cos, sin, cfg):
        C = _C()
        H, D, eps, window, f = cfg
        B, L, d = x.shape
        T = B * L
        x2 = x.reshape(T, d)
        h1, r1 = C.rms_norm_fwd(x2, wn1, eps)
        if _fuse_ok(d):
            y = ops.gemm_rope(h1, wqkv, cos, sin, L, 2 * d)
            y3 = y.view(B, L, 3 * d)
            q = y3[..., :d].view(B, L, H, D)
            k = y3[..., d:2 * d].view(B, L, H, D)
        else:
            y = ops.gemm(h1, wqkv)
            y3 = y.view(B, L, 3 * d)
            q = C.rope_fwd(y3[..., :d].view(B, L, H, D), cos, sin, False)
            k = C.rope_fwd(y3[..., d:2 * d].view(B, L, H, D), cos, sin, False)
        v = y3[..., 2 * d:].view(B, L, H, D)
        scale = D ** -0.5
        o, lse = C.attention_fwd(q, k, v, True, int(window), scale)
        x1 = ops.gemm(o.view(T, d), wout, residual=x2)
        xo, ffn_saved = _ffn_forward(x1, wn2, wfc1g, wfc2, eps, f)
        ctx.save_for_backward(x2, h1, r1, y, q, k, o, lse, x1, *ffn_saved, wn1, wqkv, wout, wn2, wfc1g, wfc2, cos,
                              sin)
        ctx.cfg = cfg
        ctx.shape = (B, L, d)
        return xo.view(B, L, d)

    @staticmethod
    def backward(ctx, dxo):
        C = _C()
        (x2, h1, r1, y, q, k, o, lse, x1, h2, r2, u, a, wn1, wqkv, wout, wn2, wfc1g, wfc2, cos,
         sin) = ctx.saved_tensors
        H, D, eps, window, f = ctx.cfg
        B, L, d = ctx.shape
        T = B * L
        dxo = dxo.reshape(T, d).contiguous()
        dx1, g_n2, g_fc1g, g_fc2 = _ffn_backward(dxo, x1, wn2, wfc1g, wfc2, (h2, r2, u, a), f)
        do = ops.gemm(dx1, wout, b_mn_major=True)
        g_out = _wgrad(wout, dx1, o.view(T, d))
        dy = torch.empty(T, 3 * d, dtype=dxo.dtype, device=dxo.device)
        dy3 = dy.view(B, L, 3 * d)
        v = y.view(B, L, 3 * d)[..., 2 * d:].view(B, L, H, D)
        C.attention_bwd(do.view(B, L, H, D), q, k, v, o, lse, True, int(window), D ** -0.5,
                        dy3[..., :d].view(B, L, H, D), dy3[..., d:2 * d].view(B, L, H, D),
                        dy3[..., 2 * d:].view(B, L, H, D), cos, sin, True, True)
        dh1 = ops.gemm(dy, wqkv, b_mn_major=True)
        g_qkv = _wgrad(wqkv, dy, h1)
        dx, dwn1 = C.rms_norm_bwd(dh1, x2, wn1, r1, dx1)
        return (dx.view(B, L, d), _ngrad(wn1, dwn1), g_qkv, g_out, g_n2, g_fc1g, g_fc2, None, None, None)


class CrossLayerFn(torch.autograd.Function):
    """x -> x + out(attention(rope(q_proj x), K, V)) -> FFN; K / V are the shared, already rotated keys/values."""

    @staticmethod
    def forward(ctx, x, K, V, wn1, wq, wout, wn2, wfc1g, wfc2, cos, sin, cfg):
        C = _C()
        Hq, D, eps, f = cfg
        B, L, d = x.shape
        T = B * L
        x2 = x.reshape(T, d)
        h1, r1 = C.rms_norm_fwd(x2, wn1, eps)
        if _fuse_ok(d):
            q = ops.gemm_rope(h1, wq, cos, sin, L, Hq * D).view(B, L, Hq, D)
        else:
            q = C.rope_fwd(ops.gemm(h1, wq).view(B, L, Hq, D), cos, sin, False)
        o, lse = C.attention_fwd(q, K, V, True, 0, D ** -0.5)
        x1 = ops.gemm(o.view(T, d), wout, residual=x2)
        xo, ffn_saved = _ffn_forward(x1, wn2, wfc1g, wfc2, eps, f)
        ctx.save_for_backward(x2, h1, r1, q, K, V, o, lse, x1, *ffn_saved, wn1, wq, wout, wn2, wfc1g, wfc2, cos, sin)
        ctx.cfg = cfg
        ctx.shape = (B, L, d)
        return xo.view(B, L, d)

    @staticmethod
    def backward(ctx, dxo):
        C = _C()
        (x2, h1, r1, q, K, V, o, lse, x1, h2, r2, u, a, wn1, wq, wout, wn2, wfc1g, wfc2, cos,
         sin) = ctx.saved_tensors
        Hq, D, eps, f = ctx.cfg
        B, L, d = ctx.shape
        T = B * L
        dxo = dxo.reshape(T, d).contiguous()
        dx1, g_n2, g_fc1g, g_fc2 = _ffn_backward(dxo, x1, wn2, wfc1g, wfc2, (h2, r2, u, a), f)
        do = ops.gemm(dx1, wout, b_mn_major=True)
        g_out = _wgrad(wout, dx1, o.view(T, d))
        dqp = torch.empty(T, d, dtype=dxo.dtype, device=dxo.device)
        _, dK, dV = C.attention_bwd(do.view(B, L, Hq, D), q, K, V, o, lse, True, 0, D ** -0.5,
                                    dqp.view(B, L, Hq, D), None, None, cos, sin, True, False)
        dh1 = ops.gemm(dqp, wq, b_mn_major=True)
        g_q = _wgrad(wq, dqp, h1)
        dx, dwn1 = C.rms_norm_bwd(dh1, x2, wn1, r1, dx1)
        return (dx.view(B, L, d), dK, dV, _ngrad(wn1, dwn1), g_q, g_out, g_n2, g_fc1g, g_fc2, None, None, None)


class SharedKVFn(torch.autograd.Function):
    """The cross-decoder's single K/V: kv_layer_norm -> kv_proj -> RoPE on K (yoco/models/decoder/yoco.py:225-239)."""

    @staticmethod
    def forward(ctx, x, wn, wkv, cos, sin, cfg):
        C = _C()
        Hk, D, eps = cfg
        B, L, d = x.shape
        T = B * L
        kvd = Hk * D
        x2 = x.reshape(T, d)
        hn, r = C.rms_norm_fwd(x2, wn, eps)
        y = ops.gemm(hn, wkv)
        y3 = y.view(B, L, 2 * kvd)
        K = C.rope_fwd(y3[..., :kvd].view(B, L, Hk, D), cos, sin, False)
        V = y3[..., kvd:].contiguous().view(B, L, Hk, D)
        ctx.save_for_backward(x2, hn, r, wn, wkv, cos, sin)
        ctx.cfg = cfg
        ctx.shape = (B, L, d)
        return K, V

    @staticmethod
    def backward(ctx, dK, dV):
        C = _C()
        x2, hn, r, wn, wkv, cos, sin = ctx.saved_tensors
        Hk, D, eps = ctx.cfg
        B, L, d = ctx.shape
        T = B * L
        kvd = Hk * D
        dy = torch.empty(T, 2 * kvd, dtype=x2.dtype, device=x2.device)
        dy[:, :kvd].copy_(C.rope_fwd(dK.contiguous(), cos, sin, True).view(T, kvd))
        dy[:, kvd:].copy_(dV.reshape(T, kvd))
        dh = ops.gemm(dy, wkv, b_mn_major=True)
        g_kv = _wgrad(wkv, dy, hn)
        dx, dwn = C.rms_norm_bwd(dh, x2, wn, r, None)
        return dx.view(B, L, d), _ngrad(wn, dwn), g_kv, None, None, None


def fused_path_ok(x: torch.Tensor, head_dim: int) -> bool:
    from ..parallel import context as CP
    from ..parallel import tp as TP
    return (ops.native_on(x) and torch.is_grad_enabled() and head_dim == 128 and x.dtype == torch.bfloat16
            and TP.tp_size() == 1 and CP.cp_size() == 1)
