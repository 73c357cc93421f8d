"""Pure-PyTorch definitions of every op the model uses.

These are the semantics the sm_100a kernels must reproduce, and they are what the model runs on CPU. Each function
states the reference expression it restates:

* RMSNorm: fp32 statistics, cast to the input dtype, then the weight multiply (yoco/models/decoder/rms_norm.py:34-46).
* Rotary embedding, interleaved (GPT-J) pairs, fp32 math on bf16 cos/sin tables
  (yoco/models/decoder/kernel/rotary.py:20-141 with interleaved=True; tables from yoco/models/decoder/yoco.py:143-152).
* SwiGLU ``x * y * sigmoid(x)`` in fp32 (yoco/models/decoder/kernel/swiglu.py:4-17).
* Gated retention: chunkwise form (yoco/models/decoder/kernel/gate_recurrent.py:204-228), the O(L^2) parallel form
  (:266-276), the decode recurrence (:253-264) and the loop oracle for the chunk-state scan (:278-288).
* Causal / sliding-window GQA attention with softmax scale 1/sqrt(head_dim) (flash_attn_func as called in
  yoco/models/decoder/cross_attention.py:42 and sliding_window_attention.py:65).
* Cross-entropy sum over non-pad targets (fairseq cross_entropy; yoco/tasks/fused_ce.py:23-59).
* Adam as apex's AdamFunctor computes it, MODE 1 = decoupled weight decay (yoco/tasks/fused_adam_cast.py:19-45).
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn.functional as F


# ----------------------------------------------------------------------------------------------------------------------
# normalisation / elementwise


def rms_norm(x: torch.Tensor, weight: Optional[torch.Tensor], eps: float) -> torch.Tensor:
    xf = x.float()
    out = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).type_as(x)
    if weight is not None:
        out = out * weight
    return out


def swiglu(x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    xf, yf = x.float(), y.float()
    return (xf * yf * torch.sigmoid(xf)).to(x.dtype)


def gate_logsigmoid(gt: torch.Tensor, normalizer: float = 16.0) -> torch.Tensor:
    return F.logsigmoid(gt) / normalizer


def llama_rope_angles(head_dim: int, max_len: int, theta: float, device=None) -> torch.Tensor:
    """The LLaMA baseline's angles: t / theta ** (arange(0, D, 2) / D) (yoco/models/decoder/transformer.py:27-31)."""
    freqs = 1.0 / (theta ** (torch.arange(0, head_dim, 2, device=device)[: head_dim // 2].float() / head_dim))
    return torch.outer(torch.arange(max_len, device=device).float(), freqs)


def rope_angles(head_dim: int, max_len: int, theta: float, device=None) -> torch.Tensor:
    """angle[t, i] = t / theta ** linspace(0, 1, head_dim // 2)[i] (note: linspace, not arange / d)."""
    angle = 1.0 / (theta ** torch.linspace(0, 1, head_dim // 2, dtype=torch.float, device=device))
    index = torch.arange(max_len, device=device).to(angle)
    return index[:, None] * angle


def rope_tables(head_dim: int, start: int, length: int, theta: float, dtype, device=None,
                angles: Optional[torch.Tensor] = None):
    if angles is None:
        angles = rope_angles(head_dim, start + length, theta, device)
    a = angles[start:start + length]
    return torch.cos(a).to(dtype), torch.sin(a).to(dtype)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, conjugate: bool = False,
               interleaved: bool = True) -> torch.Tensor:
    """x: [B, L, H, D]; cos/sin: [L, D/2]. Interleaved (GPT-J) pairs (x[2i], x[2i+1]) or, with
    ``interleaved=False``, NeoX pairs (x[i], x[i + D/2]) (yoco/models/decoder/kernel/rotary.py:302-332);
    fp32 math, output in x.dtype."""
    B, L, H, D = x.shape
    if not interleaved:
        xf = x.float()
        c = cos.float()[None, :L, None, :]
        s = sin.float()[None, :L, None, :]
        if conjugate:
            s = -s
        x0, x1 = xf[..., :D // 2], xf[..., D // 2:]
        return torch.cat([x0 * c - x1 * s, x0 * s + x1 * c], dim=-1).to(x.dtype)
    xf = x.float().view(B, L, H, D // 2, 2)
    c = cos.float()[None, :L, None, :]
    s = sin.float()[None, :L, None, :]
    if conjugate:
        s = -s
    x0, x1 = xf[..., 0], xf[..., 1]
    o0 = x0 * c - x1 * s
    o1 = x0 * s + x1 * c
    return torch.stack([o0, o1], dim=-1).view(B, L, H, D).to(x.dtype)


# ----------------------------------------------------------------------------------------------------------------------
# gated retention


def chunk_gate_recurrent_naive(kv: torch.Tensor, cross_decay: torch.Tensor, last_kv: Optional[torch.Tensor] = None):
    """Exclusive prefix states S_i = S_{i-1} * d_{i-1} + KV_{i-1}, S_0 = last_kv (or 0)."""
    B, H, N, DK, DV = kv.shape
    state = torch.zeros(B, H, DK, DV, dtype=kv.dtype, device=kv.device) if last_kv is None else last_kv
    out = []
    for i in range(N):
        out.append(state)
        state = state * cross_decay[:, :, i, None, None] + kv[:, :, i]
    return torch.stack(out, dim=2)


def chunk_gate_retention(q, k, v, g, chunk_size: int = 256, last_hidden_state=None):
    """q,k: [B,H,L,Dk], v: [B,H,L,Dv], g: [B,H,L] (log-decay per step). L must be a multiple of chunk_size."""
    bsz, num_head, tgt_len, key_dim = q.shape
    head_dim = v.shape[-1]
    n = tgt_len // chunk_size
    q = q.view(bsz, num_head, n, chunk_size, key_dim)
    k = k.view(bsz, num_head, n, chunk_size, key_dim) * (key_dim ** -0.5)
    v = v.view(bsz, num_head, n, chunk_size, head_dim)
    g = g.view(bsz, num_head, n, chunk_size).float().cumsum(-1)
    # cross-chunk part
    kv = k.transpose(-1, -2) @ (v * (-g + g[:, :, :, -1, None]).exp()[..., None].to(v.dtype))
    cross_decay = g[:, :, :, -1].exp().to(kv.dtype)
    S = chunk_gate_recurrent_naive(kv, cross_decay, last_hidden_state)
    cross = (q * g[..., None].exp().to(q.dtype)) @ S
    # intra-chunk part
    attn = q @ k.transpose(-1, -2)
    causal = torch.full([chunk_size, chunk_size], float("-inf"), device=q.device).triu(1).type_as(q)
    attn = attn * (g[..., None] - g[..., None, :] + causal).exp().to(attn.dtype)
    inner = attn @ v
    return (cross + inner).view(bsz, num_head, tgt_len, head_dim)


def hier_chunk_gate_retention(q, k, v, g, chunk_size: int = 256, hier_chunk_size: int = 16384):
    """Two-level chunking for long sequences (yoco/models/decoder/kernel/gate_recurrent.py:230-251): the sequence
    is cut into hierarchy chunks of ``hier_chunk_size``; each one is processed independently with the chunkwise form
    (state 0 at its start), and the state carried across hierarchy chunks adds ``(q exp(G_local)) @ S_prev``. Equal
    to chunk_gate_retention; the hierarchy chunks are independent units of work (e.g. one per rank or stream)."""
    B, H, L, Dk = q.shape
    Dv = v.shape[-1]
    n = L // hier_chunk_size
    if n * hier_chunk_size != L:
        raise ValueError("sequence length must be a multiple of hier_chunk_size")
    fold = lambda t, d: t.view(B, H, n, hier_chunk_size, d).transpose(1, 2).reshape(B * n, H, hier_chunk_size, d)
    inner = chunk_gate_retention(fold(q, Dk), fold(k, Dk), fold(v, Dv),
                                 g.view(B, H, n, hier_chunk_size).transpose(1, 2).reshape(B * n, H, hier_chunk_size),
                                 chunk_size)
    inner = inner.view(B, n, H, hier_chunk_size, Dv).transpose(1, 2).reshape(B, H, L, Dv)
    # hierarchy-level states: exclusive scan over the per-chunk (sum of decayed k^T v, total decay)
    qh = q.view(B, H, n, hier_chunk_size, Dk)
    kh = k.view(B, H, n, hier_chunk_size, Dk) * (Dk ** -0.5)
    vh = v.view(B, H, n, hier_chunk_size, Dv)
    G = g.view(B, H, n, hier_chunk_size).float().cumsum(-1)
    kv = kh.transpose(-1, -2) @ (vh * (G[..., -1:] - G).exp()[..., None].to(vh.dtype))
    S = chunk_gate_recurrent_naive(kv, G[..., -1].exp().to(kv.dtype))
    cross = (qh * G[..., None].exp().to(qh.dtype)) @ S
    return inner + cross.view(B, H, L, Dv)


def parallel_gate_retention(q, k, v, g):
    """O(L^2) form: o_i = sum_{j<=i} (q_i . k_j / sqrt(d)) exp(G_i - G_j) v_j with G = cumsum(g) in fp32."""
    k = k * (q.shape[-1] ** -0.5)
    L = q.shape[-2]
    causal = torch.full([L, L], float("-inf"), device=q.device).triu(1).type_as(q)
    G = g.float().cumsum(-1)
    mask = (G[..., None] - G[..., None, :] + causal).exp()
    attn = (q @ k.transpose(-1, -2)) * mask.to(q.dtype)
    return attn @ v


def parallel_gate_retention_f32(q, k, v, g):
    """The parallel form entirely in fp32 (the oracle the bf16 kernels are compared with)."""
    return parallel_gate_retention(q.float(), k.float(), v.float(), g.float())


def recurrent_gate_retention(q, k, v, g, state: Optional[torch.Tensor]):
    """One decode step. q,k: [B,H,1,Dk], v: [B,H,1,Dv], g: [B,H,1]. Returns (o, new_state)."""
    bsz, num_head, _, key_dim = q.shape
    k = k * key_dim ** -0.5
    decay = g.view(bsz, num_head, 1, 1).float().exp()
    kv = k.transpose(-1, -2) * v
    if state is not None:
        kv = kv + state * decay.to(state.dtype)
    return q @ kv, kv


def retention_prefill_state(k, v, g, index_mask: Optional[torch.Tensor], last_state: Optional[torch.Tensor]):
    """Final hidden state after a prefill block (yoco/models/decoder/gate_retention.py:86-97)."""
    head_dim = k.shape[-1]
    gf = g.float()
    if index_mask is not None:
        gf = gf.masked_fill(index_mask, 0)
    g_sum = gf.sum(dim=-1, keepdim=True)
    g_mask = (g_sum - gf.cumsum(dim=-1)).exp()
    if index_mask is not None:
        g_mask = g_mask.masked_fill(index_mask, 0)
    nxt = (k.transpose(-1, -2) * (head_dim ** -0.5)) @ (v * g_mask.to(v.dtype).unsqueeze(-1))
    if last_state is not None:
        nxt = nxt + last_state * g_sum.exp().unsqueeze(-1).to(v.dtype)
    return nxt


# ----------------------------------------------------------------------------------------------------------------------
# attention


def attention(q, k, v, causal: bool = True, window: Optional[int] = None, q_offset: int = 0,
              softmax_scale: Optional[float] = None):
    """q: [B,Lq,Hq,D], k/v: [B,Lk,Hk,D] (Hq multiple of Hk). Query i sits at absolute position q_offset + i and
    keys at 0..Lk-1; flash-attn aligns the causal diagonal to the bottom-right, which is q_offset = Lk - Lq.
    window w keeps keys j with pos_i - w < j <= pos_i (flash-attn window_size=(w-1, 0))."""
    B, Lq, Hq, D = q.shape
    Lk, Hk = k.shape[1], k.shape[2]
    scale = softmax_scale if softmax_scale is not None else D ** -0.5
    rep = Hq // Hk
    qf = q.float().transpose(1, 2)
    kf = k.float().transpose(1, 2).repeat_interleave(rep, dim=1)
    vf = v.float().transpose(1, 2).repeat_interleave(rep, dim=1)
    s = (qf @ kf.transpose(-1, -2)) * scale
    qi = torch.arange(Lq, device=q.device)[:, None] + q_offset
    kj = torch.arange(Lk, device=q.device)[None, :]
    mask = torch.zeros(Lq, Lk, dtype=torch.bool, device=q.device)
    if causal:
        mask |= kj > qi
    if window is not None:
        mask |= kj <= qi - window
    s = s.masked_fill(mask, float("-inf"))
    p = torch.softmax(s, dim=-1)
    p = torch.nan_to_num(p, nan=0.0)
    o = p @ vf
    return o.transpose(1, 2).to(q.dtype)


# ----------------------------------------------------------------------------------------------------------------------
# loss / optimizer


def cross_entropy_sum(logits: torch.Tensor, target: torch.Tensor, ignore_index: int) -> torch.Tensor:
    """fp32 sum over rows with target != ignore_index of lse(row) - row[target]."""
    lf = logits.float()
    lse = torch.logsumexp(lf, dim=-1)
    t = target.clamp_min(0)
    xt = lf.gather(-1, t[:, None]).squeeze(-1)
    loss = torch.where(target == ignore_index, torch.zeros_like(lse), lse - xt)
    return loss.sum()


def adam_step_(p: torch.Tensor, g: torch.Tensor, m: torch.Tensor, v: torch.Tensor, *, lr: float, beta1: float,
               beta2: float, eps: float, step: int, weight_decay: float, adamw: bool = True,
               bias_correction: bool = True, p16: Optional[torch.Tensor] = None):
    """In-place fp32 Adam on (p, m, v) with apex's expression; optionally writes the bf16 copy of p into p16."""
    bc1 = 1.0 - beta1 ** step if bias_correction else 1.0
    bc2 = 1.0 - beta2 ** step if bias_correction else 1.0
    bc1 = float(torch.tensor(bc1, dtype=torch.float32))
    bc2 = float(torch.tensor(bc2, dtype=torch.float32))
    g = g.float()
    if not adamw:
        g = g + weight_decay * p
    m.mul_(beta1).add_((1 - beta1) * g)
    v.mul_(beta2).add_(((1 - beta2) * g) * g)
    upd = (m / bc1) / ((v / bc2).sqrt() + eps)
    if adamw:
        upd = upd + weight_decay * p
    p.sub_(lr * upd)
    if p16 is not None:
        p16.copy_(p.to(p16.dtype))
    return p


def polynomial_decay_lr(step: int, lr: float, warmup: int, total: int, end_lr: float = 0.0,
                        power: float = 1.0) -> float:
    """fairseq polynomial_decay: linear warm-up to lr over `warmup` updates, then (lr-end)*(1-pct)^power + end."""
    if warmup > 0 and step <= warmup:
        return lr * step / float(warmup)
    if step >= total:
        return end_lr
    pct = 1 - (step - warmup) / float(total - warmup)
    return (lr - end_lr) * pct ** power + end_lr


def zero_owner_local(x: torch.Tensor, seg: int, chunk: int = 0, world: int = 1):
    """(owner, local index) of flat elements x under the ZeRO owner map: contiguous segments of ``seg`` elements
    (chunk 0), or chunks of ``chunk`` elements dealt to ``world`` ranks in turn."""
    if chunk:
        return (x // chunk) % world, (x // (chunk * world)) * chunk + x % chunk
    o = torch.div(x, seg, rounding_mode="floor")
    return o, x - o * seg


def owner_scatter(dw: torch.Tensor, x0: int, seg: int, rank: int, own: torch.Tensor, staging, chunk: int = 0) -> None:
    """Where the GEMM-fused ZeRO reduce-scatter stores a weight gradient computed on ``rank``: element i of
    ``dw.reshape(-1)`` has flat index x = x0 + i, owner o and local index l (``zero_owner_local``); it goes to
    ``own[x]`` when o == rank, else to ``staging[o][rank * seg + l]`` (owner o's slot for this rank)."""
    flat = dw.reshape(-1)
    x = torch.arange(x0, x0 + flat.numel(), device=flat.device)
    o, loc = zero_owner_local(x, seg, chunk, len(staging))
    mine = o == rank
    own[x[mine]] = flat[mine].to(own.dtype)
    for q in torch.unique(o[~mine]).tolist():
        m = o == q
        staging[q][rank * seg + loc[m]] = flat[m].to(staging[q].dtype)


def staged_owner_sum(own: torch.Tensor, staging: torch.Tensor, rank: int, world: int, seg: int, lo: int,
                     n: int) -> torch.Tensor:
    """The owner's reduction of [lo, lo + n) of its segment: fp32 sum over ranks in rank order (its own values from
    its gradient buffer, the others' from staging slot r), divided by world, rounded to bf16."""
    loc = lo - rank * seg
    acc = torch.zeros(n, dtype=torch.float32, device=own.device)
    for r in range(world):
        src = own[lo:lo + n] if r == rank else staging[r * seg + loc: r * seg + loc + n]
        acc += src.float()
    return (acc * (1.0 / world)).to(torch.bfloat16)
