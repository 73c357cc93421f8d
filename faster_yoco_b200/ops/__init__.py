"""Public op API of the framework.

Every op has two implementations behind one signature:

* ``native`` (default on CUDA tensors): the sm_100a kernels of ``faster_yoco_b200/csrc`` through the in-tree
  extension. A missing extension raises; there is no silent fallback on a GPU.
* ``torch``: the reference expressions of :mod:`faster_yoco_b200.ops.reference` run by PyTorch (cuBLAS GEMMs,
  flash-attn / SDPA attention). This is the in-repo baseline that the native path is compared with, and the path
  every op takes on CPU tensors.

The backend is a process-wide setting (``set_backend``), not a per-call dispatch.
"""
from __future__ import annotations

import math
import os
from typing import Optional

import torch
import torch.nn.functional as F

from . import reference as ref
from . import _native

_BACKEND = "native"


def set_backend(name: str):
    global _BACKEND
    if name not in ("native", "torch"):
        raise ValueError(name)
    _BACKEND = name


def get_backend() -> str:
    return _BACKEND


def native_on(t: torch.Tensor) -> bool:
    return t.is_cuda and _BACKEND == "native"


def _C():
    return _native.lib()


# CTA-pair kernel (gemm2.cu) for large GEMMs: on by default (68.6 vs 71.2 ms per YOCO-3B update on one B200);
# FYB_GEMM_PAIR=0 keeps every GEMM on the one-CTA kernel
_GEMM_PAIR = os.environ.get("FYB_GEMM_PAIR", "1") == "1"


def _grad_slot(p):
    """(slot, accumulate) when p lives in a flat ZeRO buffer that takes gradients directly, else (None, False)."""
    fp = getattr(p, "_fyb_flat", None)
    if fp is None or not fp.direct_grads:
        return None, False
    return fp.claim_grad(p)


def wgrad_into(w: torch.Tensor, dy: torch.Tensor, x: torch.Tensor) -> bool:
    """dW = dy^T x (dy [T, N], x [T, K]) written into w's flat gradient slot; False when w has no slot.

    With the GEMM-fused reduce-scatter on (``FlatParams.scatter``), the GEMM's epilogue stores every element at
    its ZeRO owner instead (this rank's slot for the rows it owns, the owner's staging buffer over NVLink for the
    others), so no separate gradient exchange pass reads the slot again."""
    fp = getattr(w, "_fyb_flat", None)
    if fp is None or not fp.direct_grads:
        return False
    slot, acc = fp.claim_grad(w)
    if fp.scatter is not None and slot.numel() % 8 == 0 and w.shape[-1] % 8 == 0:
        bases = fp.scatter_target(w)
        if bases is not None:
            _C().gemm_scatter(dy, x, slot, acc, fp.grad_flat, bases, fp.seg, fp.rank, fp.chunk)
            return True
    if fp.sq_mode:
        part = fp.sq_partials(w)
        if part is not None:
            # the GEMM also writes the sum of squares of the stored gradient (one-GPU gradient norm, no extra pass)
            fp.sq_commit(w, int(_C().gemm_sq(dy, x, slot, acc, part)))
            return True
    gemm(dy, x, a_mn_major=True, b_mn_major=True, out=slot, residual=slot if acc else None)
    return True


# ----------------------------------------------------------------------------------------------------------------------
# GEMM: y = x @ w.T (+ residual)


def gemm(a: torch.Tensor, b: torch.Tensor, *, a_mn_major: bool = False, b_mn_major: bool = False,
         out: Optional[torch.Tensor] = None, residual: Optional[torch.Tensor] = None,
         out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """C[M,N] = sum_k A(m,k) B(n,k) on the tcgen05 GEMM.

    A is stored [M,K] (K-major) or [K,M] (``a_mn_major``); B is stored [N,K] or [K,N] (``b_mn_major``)."""
    M = a.shape[1] if a_mn_major else a.shape[0]
    N = b.shape[1] if b_mn_major else b.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=out_dtype or a.dtype, device=a.device)
    K = a.shape[0] if a_mn_major else a.shape[1]
    if not a_mn_major and not b_mn_major and out.dtype == torch.bfloat16:
        pa = _pull_args(b)
        if pa is not None:
            # the weight's all-gather runs inside this (its first forward) GEMM
            _C().gemm_gather(a, b, out, *pa, _gather_bn(M, N, K), None, None, 0, 0, residual)
            return out
    route = _gemm_route(M, N, K) if _GEMM_PAIR else (0, 0, 1)
    if route[0] == 1:
        _C().gemm_pair(a, b, out, a_mn_major, b_mn_major, residual, route[1], route[2])
    else:
        _C().gemm(a, b, out, a_mn_major, b_mn_major, residual)
    return out


_ROUTES = {}


def _pull_args(w: torch.Tensor):
    """Gather-GEMM arguments when w's ZeRO all-gather runs inside the GEMM that first reads it this update."""
    fp = getattr(w, "_fyb_flat", None)
    if fp is None or fp.pull is None:
        return None
    return fp.pull_args(w)


def _gather_bn(M: int, N: int, K: int) -> int:
    route = _gemm_route(M, N, K)
    return 192 if route[0] == 1 and route[1] == 192 and route[2] == 1 else 256


def _gemm_route(M: int, N: int, K: int):
    """(kernel, tile width, splits) for the shape from the cost model of csrc/gemm.cu::gemm_route (cached per
    shape)."""
    key = (M, N, K)
    r = _ROUTES.get(key)
    if r is None:
        r = _ROUTES[key] = tuple(_C().gemm_route(M, N, K))
    return r


# Elementwise epilogues of the CTA-pair GEMM (csrc/gemm2.cu): the rotary embedding of the q / k blocks in the
# projection that produces them, SwiGLU in the merged fc1 | gate projection and the SwiGLU backward in the fc2 input
# gradient. Each saves one read + write of an activation and a launch per layer. FYB_GEMM_FUSE=0 runs the GEMM and
# the elementwise kernel separately (same values; comparison switch).
GEMM_FUSE = os.environ.get("FYB_GEMM_FUSE", "1") == "1"


def gemm_rope(a: torch.Tensor, w: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, seq_len: int, rot_cols: int,
              out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = a @ w.T with the interleaved rotary embedding (head dim 128) applied to columns [0, rot_cols) of every
    row, row r at position r mod seq_len -- the values of gemm() followed by rope() on those head blocks.
    a: [T, K]; w: [N, K]; cos / sin: the [>= seq_len, 64] tables of ``rope``."""
    T, N = a.shape[0], w.shape[0]
    if out is None:
        out = torch.empty(T, N, dtype=a.dtype, device=a.device)
    if native_on(a):
        pa = _pull_args(w)
        if pa is not None:
            _C().gemm_gather(a, w, out, *pa, _gather_bn(T, N, a.shape[1]), cos, sin, seq_len, rot_cols)
            return out
        route = _gemm_route(T, N, a.shape[1])
        bn = route[1] if route[0] == 1 and route[2] == 1 else 256
        _C().gemm_rope(a, w, out, cos, sin, seq_len, rot_cols, bn)
        return out
    y = gemm(a, w, out=out)
    if rot_cols:
        blk = y[:, :rot_cols].view(T // seq_len, seq_len, rot_cols // 128, 128)
        blk.copy_(ref.apply_rope(blk, cos[:seq_len], sin[:seq_len]))
    return out


def gemm_swiglu(a: torch.Tensor, w: torch.Tensor):
    """(u, h): u = a @ w.T for the merged [fc1; gate] weight w [2f, K], h = silu(u[:, :f]) * u[:, f:] -- one GEMM
    whose epilogue also computes the activation (values of gemm() followed by swiglu())."""
    if native_on(a):
        pa = _pull_args(w)
        if pa is not None:
            u, h = _C().gemm_gather_swiglu(a, w, *pa)
        else:
            u, h = _C().gemm_swiglu(a, w)
        return u, h
    u = gemm(a, w)
    f = u.shape[1] // 2
    return u, ref.swiglu(u[:, :f], u[:, f:])


def gemm_swiglu_bwd(g: torch.Tensor, w2: torch.Tensor, u: torch.Tensor, du: Optional[torch.Tensor] = None):
    """du = [da | db], the SwiGLU backward of dh = g @ w2 (w2: the fc2 weight [d, f], g: [T, d]) against the saved
    fc1 | gate output u [T, 2f], with dh never stored (values of gemm() followed by the swiglu backward)."""
    if du is None:
        du = torch.empty_like(u)
    if native_on(g):
        _C().gemm_swiglu_bwd(g, w2, True, u, du)
        return du
    dh = gemm(g, w2, b_mn_major=True)
    f = u.shape[1] // 2
    a32, b32 = u[:, :f].float(), u[:, f:].float()
    s = torch.sigmoid(a32)
    du[:, :f] = (s * (1 + a32 * (1 - s)) * dh.float() * b32).to(du.dtype)
    du[:, f:] = (a32 * s * dh.float()).to(du.dtype)
    return du


def gemm_gather(a: torch.Tensor, w: torch.Tensor, flat: torch.Tensor, peers: torch.Tensor, seg: int, chunk: int,
                rank: int, out: Optional[torch.Tensor] = None, rope=None) -> torch.Tensor:
    """y = a @ w.T with the ZeRO parameter all-gather of w fused into the GEMM: w is a contiguous weight inside this
    rank's flat replica `flat`; its rows owned by other ranks (owner map seg / chunk) are pulled from the owners'
    replicas (`peers`: device int64 [world] base addresses) by the GEMM's gather warps ahead of the tiles that read
    them, so w is current in this replica on return. rope: optional (cos, sin, seq_len, rot_cols) as gemm_rope.
    No torch form: the peer replicas are device memory of other GPUs."""
    T, N = a.shape[0], w.shape[0]
    if out is None:
        out = torch.empty(T, N, dtype=a.dtype, device=a.device)
    bn = _gather_bn(T, N, a.shape[1])
    if rope is None:
        _C().gemm_gather(a, w, out, flat, peers, seg, chunk, rank, bn)
    else:
        cos, sin, seq_len, rot_cols = rope
        _C().gemm_gather(a, w, out, flat, peers, seg, chunk, rank, bn, cos, sin, seq_len, rot_cols)
    return out


class _NativeLinear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, residual):
        shp = x.shape
        x2 = x.reshape(-1, shp[-1])
        r2 = residual.reshape(-1, w.shape[0]) if residual is not None else None
        y = gemm(x2, w, residual=r2)
        ctx.save_for_backward(x2, w)
        ctx.shp = shp
        ctx.has_res = residual is not None
        return y.view(*shp[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, w = ctx.saved_tensors
        dy2 = dy.reshape(-1, w.shape[0])
        if not dy2.is_contiguous():
            dy2 = dy2.contiguous()
        dx = dw = None
        if ctx.needs_input_grad[0]:
            dx = gemm(dy2, w, b_mn_major=True).view(ctx.shp)
        if ctx.needs_input_grad[1]:
            # the weight gradient lands in the flat gradient buffer (or at its owners); autograd sees none for w
            if not wgrad_into(w, dy2, x2):
                dw = gemm(dy2, x2, a_mn_major=True, b_mn_major=True)
        return dx, dw, (dy if ctx.has_res else None)


def linear(x: torch.Tensor, w: torch.Tensor, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = x @ w.T (+ residual). The tcgen05 GEMM needs 16-byte aligned rows (K and N multiples of 8 bf16);
    other shapes (e.g. LLaMA's int(8 d / 3) FFN width) run on cuBLAS."""
    if native_on(x) and x.shape[-1] % 8 == 0 and w.shape[0] % 8 == 0 and x.dtype == torch.bfloat16:
        return _NativeLinear.apply(x, w, residual)
    y = F.linear(x, w)
    return y + residual if residual is not None else y


# ----------------------------------------------------------------------------------------------------------------------
# RMSNorm


class _NativeRMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        shp = x.shape
        x2 = x.reshape(-1, shp[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        y, rstd = _C().rms_norm_fwd(x2, w, float(eps))
        ctx.save_for_backward(x2, w, rstd)
        ctx.shp = shp
        return y.view(shp)

    @staticmethod
    def backward(ctx, dy):
        x2, w, rstd = ctx.saved_tensors
        dy2 = dy.reshape(x2.shape)
        if not dy2.is_contiguous():
            dy2 = dy2.contiguous()
        dx, dw = _C().rms_norm_bwd(dy2, x2, w, rstd)
        if w is not None:
            slot, acc = _grad_slot(w)
            if slot is not None:
                slot.add_(dw) if acc else slot.copy_(dw)
                dw = None
        return dx.view(ctx.shp), (dw if w is not None else None), None


def rms_norm(x: torch.Tensor, weight: Optional[torch.Tensor], eps: float) -> torch.Tensor:
    if native_on(x) and x.dtype == torch.bfloat16 and x.shape[-1] % 8 == 0:
        return _NativeRMSNorm.apply(x, weight, eps)
    return ref.rms_norm(x, weight, eps)


# ----------------------------------------------------------------------------------------------------------------------
# SwiGLU


class _NativeSwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, y):
        out = _C().swiglu_fwd(x, y)
        ctx.save_for_backward(x, y)
        return out

    @staticmethod
    def backward(ctx, dout):
        x, y = ctx.saved_tensors
        dx, dy = _C().swiglu_bwd(x, y, dout.contiguous())
        return dx, dy


def _rows16(t: torch.Tensor) -> bool:
    """bf16 rows of a multiple of 8 elements on 16-byte boundaries (the vector width of the elementwise kernels)."""
    return (t.dtype == torch.bfloat16 and t.shape[-1] % 8 == 0 and t.stride(-1) == 1
            and all(st % 8 == 0 for st in t.stride()[:-1]) and t.data_ptr() % 16 == 0)


def swiglu(x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    """x * y * sigmoid(x) (silu on the FIRST argument, as the reference's kernel/swiglu.py). Rows that are not
    16-byte vectors (e.g. LLaMA's int(8 d / 3) width) take the PyTorch expression."""
    if native_on(x) and _rows16(x) and _rows16(y):
        shp = x.shape
        return _NativeSwiGLU.apply(x.reshape(-1, shp[-1]), y.reshape(-1, shp[-1])).view(shp)
    return ref.swiglu(x, y)


# ----------------------------------------------------------------------------------------------------------------------
# rotary embedding (interleaved)


class _NativeRope(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, cos, sin, neox):
        ctx.save_for_backward(cos, sin)
        ctx.neox = neox
        return _C().rope_fwd(x, cos, sin, False, neox)

    @staticmethod
    def backward(ctx, dy):
        cos, sin = ctx.saved_tensors
        if dy.stride(-1) != 1 or any(st % 8 for st in dy.stride()[:-1]):
            dy = dy.contiguous()
        return _C().rope_fwd(dy, cos, sin, True, ctx.neox), None, None, None


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, interleaved: bool = True) -> torch.Tensor:
    """x: [B, L, H, D] (any strides with a contiguous last dim); returns a contiguous [B, L, H, D].
    ``interleaved=False`` rotates NeoX half pairs (the LLaMA baseline's mode)."""
    if native_on(x) and (interleaved or x.size(-1) % 16 == 0):
        if x.stride(-1) != 1 or any(st % 8 for st in x.stride()[:-1]):
            x = x.contiguous()
        return _NativeRope.apply(x, cos, sin, not interleaved)
    return ref.apply_rope(x, cos, sin, interleaved=interleaved)


# ----------------------------------------------------------------------------------------------------------------------
# per-head weightless RMSNorm (subln) fused with the output gate swiglu(g, .)


class _NativeSublnSwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, o, g, eps, head_dim):
        out, rstd = _C().subln_swiglu_fwd(o, g, float(eps), int(head_dim))
        ctx.save_for_backward(o, g, rstd)
        ctx.head_dim = head_dim
        return out

    @staticmethod
    def backward(ctx, dout):
        o, g, rstd = ctx.saved_tensors
        do, dg = _C().subln_swiglu_bwd(dout.contiguous(), o, g, rstd, int(ctx.head_dim))
        return do, dg, None, None


def subln_swiglu(o: torch.Tensor, g: torch.Tensor, eps: float, head_dim: int) -> torch.Tensor:
    """o: [T, H*D] retention output (token-major); g: [T, H*D]. Returns swiglu(g, rmsnorm_per_head(o))."""
    if native_on(o):
        return _NativeSublnSwiGLU.apply(o, g, eps, head_dim)
    T, HD = o.shape
    on = ref.rms_norm(o.view(T, HD // head_dim, head_dim), None, eps).view(T, HD)
    return ref.swiglu(g, on)


# ----------------------------------------------------------------------------------------------------------------------
# gated retention


def gate_logsigmoid(gt: torch.Tensor, normalizer: float) -> torch.Tensor:
    return F.logsigmoid(gt) / normalizer


# FYB_RETENTION=parallel: the quadratic parallel-form kernel (attention.cu) instead of the chunkwise kernels
# (retention.cu); kept as a second implementation for comparison
RETENTION_FORM = os.environ.get("FYB_RETENTION", "chunk")


class _NativeRetention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, gcum):
        o = _C().retention_fwd(q, k, v, gcum)
        ctx.save_for_backward(q, k, v, gcum, o)
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, gcum, o = ctx.saved_tensors
        dq, dk, dv, dg = _C().retention_bwd(do.contiguous(), q, k, v, gcum, o)
        return dq, dk, dv, dg


class _NativeChunkRetention(torch.autograd.Function):
    """Chunkwise retention (retention.cu) on the per-step log decays g [B, H, L] (fp32): the kernels see the
    chunk-local cumsum; the gate gradient comes back w.r.t. the global cumsum G, so dL/dg = reverse cumsum of it."""

    @staticmethod
    def forward(ctx, q, k, v, g):
        C = _C()
        gloc = C.retention_chunk_cumsum(g)
        o, states, _ = C.retention_chunk_fwd(q, k, v, gloc)
        ctx.save_for_backward(q, k, v, gloc, states)
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, gloc, states = ctx.saved_tensors
        dq, dk, dv, _, dG = _C().retention_chunk_bwd(do.contiguous(), q, k, v, gloc, states, want_dgate=True)
        dg = dG.flip(-1).cumsum(-1).flip(-1)
        return dq, dk, dv, dg


def retention_prefill(q, k, v, g, state=None, index_mask=None):
    """Chunked prefill on the GPU: outputs of a block of L tokens and the state after it.

    q, k, v: [B, L, H, 128] bf16; g: [B, L, H] per-step log decays; state: fp32 [B, H, 128, 128] entering the block
    (or None). index_mask: optional bool [B, H, L] (True = padding), applied to the state only, as the reference's
    prefill does (outputs use every position). Returns (o [B, L, H, 128], new fp32 state)."""
    C = _C()
    gh = g.float().transpose(1, 2).contiguous()
    gloc = C.retention_chunk_cumsum(gh)
    st = state.float().contiguous() if state is not None else None
    if index_mask is None:
        o, _, nxt = C.retention_chunk_fwd(q, k, v, gloc, state_in=st, want_state=True)
        return o, nxt
    o, _, _ = C.retention_chunk_fwd(q, k, v, gloc, state_in=st)
    index_mask = torch.broadcast_to(index_mask.to(q.device), gh.shape)
    keep = (~index_mask).transpose(1, 2).unsqueeze(-1)                 # [B, L, H, 1]
    km = (k * keep.to(k.dtype)).contiguous()
    gm = C.retention_chunk_cumsum(gh.masked_fill(index_mask, 0.0).contiguous())
    return o, C.retention_chunk_state(km, v, gm, state_in=st)


def retention_decode(q, k, v, g, state):
    """One decode step: q, k, v [B, 1, H, 128] bf16, g [B, 1, H] log decays, state fp32 [B, H, 128, 128] (updated in
    place). Returns o [B, 1, H, 128]."""
    o = _C().retention_decode(q[:, 0], k[:, 0], v[:, 0], g[:, 0].float().contiguous(), state)
    return o.unsqueeze(1)


def retention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, gt: torch.Tensor,
              chunk_size: int = 256) -> torch.Tensor:
    """Gated retention over a full sequence (training path).

    q, k, v: [B, L, H, D] (token-major, any strides with a contiguous last dim); gt: [B, L, H] per-step log decay
    (logsigmoid / normalizer, any float dtype). Returns o: [B, L, H, D] contiguous."""
    B, L, H, D = q.shape
    if native_on(q) and D == 128:
        if RETENTION_FORM == "parallel":
            gcum = gt.float().transpose(1, 2).cumsum(-1).contiguous()      # [B, H, L] fp32
            return _NativeRetention.apply(q, k, v, gcum)
        return _NativeChunkRetention.apply(q, k, v, gt.float().transpose(1, 2).contiguous())
    qh, kh, vh = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    gh = gt.transpose(1, 2)
    if L % chunk_size == 0:
        o = ref.chunk_gate_retention(qh, kh, vh, gh, chunk_size=chunk_size)
    else:
        o = ref.parallel_gate_retention(qh, kh, vh, gh)
    return o.transpose(1, 2).contiguous()


# ----------------------------------------------------------------------------------------------------------------------
# attention (causal / sliding window, GQA)


class _NativeAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal, window, scale):
        o, lse = _C().attention_fwd(q, k, v, bool(causal), int(window or 0), float(scale))
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.cfg = (bool(causal), int(window or 0), float(scale))
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        causal, window, scale = ctx.cfg
        dq, dk, dv = _C().attention_bwd(do.contiguous(), q, k, v, o, lse, causal, window, scale)
        return dq, dk, dv, None, None, None


_flash_attn_func = None


def _flash():
    global _flash_attn_func
    if _flash_attn_func is None:
        try:
            from flash_attn import flash_attn_func
            _flash_attn_func = flash_attn_func
        except Exception:
            _flash_attn_func = False
    return _flash_attn_func


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = True,
              window: Optional[int] = None) -> torch.Tensor:
    """q: [B, Lq, Hq, D], k/v: [B, Lk, Hk, D] -> [B, Lq, Hq, D]; scale 1/sqrt(D); window as flash-attn (w-1, 0)."""
    scale = q.shape[-1] ** -0.5
    if native_on(q) and q.shape[-1] == 128:
        return _NativeAttention.apply(q, k, v, causal, window, scale)
    if q.is_cuda and q.dtype in (torch.float16, torch.bfloat16) and _flash():
        ws = (window - 1, 0) if window is not None else (-1, -1)
        return _flash()(q, k, v, causal=causal, window_size=ws)
    return ref.attention(q, k, v, causal=causal, window=window, q_offset=k.shape[1] - q.shape[1])


# ----------------------------------------------------------------------------------------------------------------------
# token embedding (x scale)


class _NativeEmbedding(torch.autograd.Function):
    @staticmethod
    def forward(ctx, tokens, w, scale):
        out = _C().embedding_fwd(tokens, w, float(scale))
        ctx.save_for_backward(tokens)
        ctx.vshape = w.shape
        ctx.scale = scale
        ctx.param = w
        return out

    @staticmethod
    def backward(ctx, dy):
        (tokens,) = ctx.saved_tensors
        slot, acc = _grad_slot(ctx.param)
        dy2 = dy.reshape(-1, ctx.vshape[1]).contiguous()
        if slot is not None and not acc:
            fp = ctx.param._fyb_flat
            bases = fp.sparse_target(ctx.param) if fp.scatter is not None and ctx.vshape[1] % 8 == 0 else None
            if bases is not None:
                # GEMM-fused reduce-scatter on: the rows of this batch's tokens go straight to their owners
                _C().embedding_bwd_scatter(tokens.reshape(-1), dy2, float(ctx.scale), slot, fp.grad_flat, bases,
                                           fp.seg, fp.rank, fp.chunk)
                return None, None, None
            _C().embedding_bwd(tokens, dy2, int(ctx.vshape[0]), float(ctx.scale), slot)
            return None, None, None
        dw = _C().embedding_bwd(tokens, dy2, int(ctx.vshape[0]), float(ctx.scale), None)
        if slot is not None:
            slot.add_(dw)
            return None, None, None
        return None, dw, None


def embedding(tokens: torch.Tensor, w: torch.Tensor, scale: float) -> torch.Tensor:
    if native_on(w):
        shp = tokens.shape
        return _NativeEmbedding.apply(tokens.reshape(-1), w, scale).view(*shp, w.shape[1])
    return scale * F.embedding(tokens, w)


# ----------------------------------------------------------------------------------------------------------------------
# cross-entropy over the vocabulary


class _NativeCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, target, ignore_index):
        loss_rows, lse = _C().ce_fwd(logits, target, int(ignore_index))
        ctx.save_for_backward(logits, target, lse)
        ctx.ignore = int(ignore_index)
        return loss_rows.sum()

    @staticmethod
    def backward(ctx, grad):
        logits, target, lse = ctx.saved_tensors
        g = grad.reshape(1).float().contiguous()
        # the logits are not needed after this: the gradient overwrites them in place
        dx = _C().ce_bwd(logits, target, lse, g, ctx.ignore, logits)
        return dx, None, None


def cross_entropy(logits: torch.Tensor, target: torch.Tensor, ignore_index: int) -> torch.Tensor:
    """fp32 sum over non-ignored rows of lse - logit[target]. logits [N, V] (bf16), target [N] int64."""
    if native_on(logits):
        return _NativeCE.apply(logits, target, ignore_index)
    lp = F.log_softmax(logits.float(), dim=-1)
    return F.nll_loss(lp, target, ignore_index=ignore_index, reduction="sum")


__all__ = [
    "set_backend", "get_backend", "gemm", "linear", "rms_norm", "swiglu", "rope", "subln_swiglu", "gate_logsigmoid",
    "retention", "retention_prefill", "retention_decode", "attention", "embedding", "cross_entropy", "ref",
]
