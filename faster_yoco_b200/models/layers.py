"""Building blocks of the YOCO decoder: RMSNorm, the three token mixers and the SwiGLU FFN.

Layout decisions (B200-first, not the reference's): the projections that read the same input are ONE parameter,
physically contiguous, so each is one GEMM with no per-step ``torch.cat`` (the reference concatenates the q/k/v/g
weights every forward under YOCO_FUSE_QKVG, yoco/models/decoder/gate_retention.py:61-66):

* gated retention: ``qkvg_proj`` = rows [q | k | v | g | gt | zero pad to a multiple of 8]
* sliding-window attention: ``qkv_proj`` = [q | k | v]
* FFN: ``fc1_gate`` = [fc1 | gate]
* cross-decoder shared KV: ``kv_proj`` = [k | v]

State dicts are written and read with the reference's per-projection names (``mixer.q_proj.weight`` ...) by the
hooks in :mod:`faster_yoco_b200.models.yoco`.

Tensor parallelism (``model_parallel_size`` > 1, after ``parallel.tp.init_model_parallel``) follows the reference's
Megatron declarations (gate_retention.py:40-46, feedforward_network.py:24-26, cross_attention.py, decoder/yoco.py):
every input projection is column-parallel (each rank holds its heads / its FFN columns of EVERY merged part),
every output projection is row-parallel (partial products summed across the TP group before the residual add), the
embedding is vocabulary-parallel and the output projection column-parallel with gathered logits. Master weights are
initialised in full and sliced, so a TP run starts from the TP=1 weights.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from .. import ops
from ..parallel import context as CP
from ..parallel import tp as TP
from . import init as I


def _tp() -> int:
    return TP.tp_size()


def _slice_rows(full: torch.Tensor) -> torch.Tensor:
    n = full.shape[0] // _tp()
    return full[TP.tp_rank() * n:(TP.tp_rank() + 1) * n]


def _slice_cols(full: torch.Tensor) -> torch.Tensor:
    n = full.shape[1] // _tp()
    return full[:, TP.tp_rank() * n:(TP.tp_rank() + 1) * n]


def _round8(n: int) -> int:
    return (n + 7) // 8 * 8


class RMSNorm(nn.Module):
    """x * rsqrt(mean(x^2) + eps) in fp32, cast back, times weight (yoco/models/decoder/rms_norm.py:23-49)."""

    def __init__(self, dim: int, eps: float = 1e-6, elementwise_affine: bool = True):
        super().__init__()
        self.dim, self.eps, self.elementwise_affine = dim, eps, elementwise_affine
        if elementwise_affine:
            self.weight = nn.Parameter(torch.ones(dim))
        else:
            self.register_parameter("weight", None)

    def forward(self, x):
        return ops.rms_norm(x, self.weight, self.eps)

    def extra_repr(self):
        return f"dim={self.dim}, eps={self.eps}, elementwise_affine={self.elementwise_affine}"


class MergedLinear(nn.Module):
    """One weight [sum(parts) (+pad), in] whose row blocks are the logical projections ``names``. Under tensor
    parallelism every part is column-split: this rank keeps rows [rank * n / tp, (rank + 1) * n / tp) of each."""

    def __init__(self, in_features: int, parts, names, inits, pad_to8: bool = False):
        super().__init__()
        self.in_features = in_features
        self.full_parts = list(parts)
        tp = _tp()
        if any(n % tp for n in self.full_parts):
            raise ValueError(f"merged projection parts {self.full_parts} not divisible by TP size {tp}")
        self.parts = [n // tp for n in self.full_parts]
        self.names = list(names)
        rows = sum(self.parts)
        self.rows = _round8(rows) if pad_to8 else rows
        self.weight = TP.mark_sharded(nn.Parameter(torch.empty(self.rows, in_features)))
        self._inits = list(inits)
        self.reset_parameters()

    def reset_parameters(self, init_override=None):
        with torch.no_grad():
            self.weight.zero_()
            off = 0
            for n_full, n, f in zip(self.full_parts, self.parts, self._inits):
                if _tp() == 1:
                    (init_override or f)(self.weight[off:off + n])
                else:
                    full = torch.empty(n_full, self.in_features, device=self.weight.device)
                    (init_override or f)(full)
                    self.weight[off:off + n].copy_(_slice_rows(full))
                off += n

    def offsets(self):
        off, out = 0, []
        for n in self.parts:
            out.append((off, n))
            off += n
        return out

    def forward(self, x, residual=None):
        return ops.linear(x, self.weight, residual)


class Linear(nn.Module):
    """``parallel``: None (replicated), "column" (output features split across the TP group) or "row" (input
    features split; the partial products are summed across the group before the residual is added)."""

    def __init__(self, in_features: int, out_features: int, init=I.init_method, parallel: Optional[str] = None):
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        self.parallel = parallel if _tp() > 1 else None
        shape = [out_features, in_features]
        if self.parallel == "column":
            shape[0] //= _tp()
        elif self.parallel == "row":
            shape[1] //= _tp()
        self.weight = nn.Parameter(torch.empty(*shape))
        if self.parallel is not None:
            TP.mark_sharded(self.weight)
        self._init = init
        self.reset_parameters()

    def reset_parameters(self, init_override=None):
        with torch.no_grad():
            fn = init_override or self._init
            if self.parallel is None:
                fn(self.weight)
                return
            full = torch.empty(self.out_features, self.in_features, device=self.weight.device)
            fn(full)
            self.weight.copy_(_slice_rows(full) if self.parallel == "column" else _slice_cols(full))

    def forward(self, x, residual=None):
        if self.parallel == "row":
            y = TP.reduce_from_tp(ops.linear(x, self.weight))
            return y + residual if residual is not None else y
        return ops.linear(x, self.weight, residual)


class FeedForwardNetwork(nn.Module):
    """fc2(swiglu(fc1 x, gate x)) with silu on fc1 (yoco/models/decoder/feedforward_network.py:15-33)."""

    def __init__(self, embed_dim: int, ffn_dim: int):
        super().__init__()
        self.embed_dim, self.ffn_dim = embed_dim, ffn_dim
        self.fc1_gate = MergedLinear(embed_dim, [ffn_dim, ffn_dim], ["fc1", "gate"], [I.init_method, I.init_method])
        self.fc2 = Linear(ffn_dim, embed_dim, I.init_method, parallel="row")

    def forward(self, x, residual=None):
        h = self.fc1_gate(TP.copy_to_tp(x))
        f = self.fc1_gate.parts[0]
        a = ops.swiglu(h[..., :f], h[..., f:])
        return self.fc2(a, residual)


class GateRetention(nn.Module):
    """Gated retention mixer (yoco/models/decoder/gate_retention.py:27-109).

    q/k/v/g: d -> d, gt: d -> n_heads; RoPE (interleaved) on q and k; gt = logsigmoid(gt) / 16; keys scaled by
    head_dim^-0.5 inside the retention op; weightless per-head RMSNorm (subln) of the output, then swiglu(g, o), then
    out_proj."""

    def __init__(self, args):
        super().__init__()
        self.args = args
        self.embed_dim = args.dim
        self.num_heads = args.n_self_heads // args.model_parallel_size
        self.head_dim = args.dim // args.n_self_heads
        d = args.dim
        self.qkvg_proj = MergedLinear(d, [d, d, d, d, args.n_self_heads], ["q_proj", "k_proj", "v_proj", "g_proj",
                                                                           "gt_proj"],
                                      [I.qkvg_init_method] * 5, pad_to8=True)
        self.out_proj = Linear(d, d, I.out_init_method, parallel="row")
        self.subln_eps = args.norm_eps
        self.gate_logit_normalizer = args.gate_logit_normalizer

    def project(self, x):
        B, L, _ = x.shape
        H, D = self.num_heads, self.head_dim
        d = H * D                                   # this rank's width (the full width without TP)
        y = self.qkvg_proj(TP.copy_to_tp(x))
        q = y[..., 0 * d:1 * d].view(B, L, H, D)
        k = y[..., 1 * d:2 * d].view(B, L, H, D)
        v = y[..., 2 * d:3 * d].view(B, L, H, D)
        g = y[..., 3 * d:4 * d]
        gt = y[..., 4 * d:4 * d + H]
        return q, k, v, g, gt

    def forward(self, x, rel_pos, incremental_state=None, is_prefilling=False, residual=None):
        B, L, _ = x.shape
        H, D = self.num_heads, self.head_dim
        q, k, v, g, gt = self.project(x)
        cos, sin = rel_pos
        q = ops.rope(q, cos, sin)
        k = ops.rope(k, cos, sin)
        gt = ops.gate_logsigmoid(gt, self.gate_logit_normalizer)            # [B, L, H]
        if incremental_state is not None and not is_prefilling:
            o = self._decode(q, k, v, gt, incremental_state)
        elif incremental_state is not None:
            o = self._prefill(q, k, v, gt, incremental_state)
        else:
            o = ops.retention(q, k, v, gt, chunk_size=self.args.chunk_size)      # [B, L, H, D]
            if CP.cp_size() > 1:       # state carried in from the earlier sequence blocks of the group
                carry = CP.retention_carry(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                           gt.transpose(1, 2))
                o = o + carry.transpose(1, 2).to(o.dtype)
        o = ops.subln_swiglu(o.reshape(B * L, H * D), g.reshape(B * L, H * D), self.subln_eps, D)
        o = o.view(B, L, H * D)
        return self.out_proj(o, residual)

    # inference paths (yoco/models/decoder/gate_retention.py:83-97): on the GPU the chunkwise prefill and the decode
    # step are native kernels (fp32 state); elsewhere the PyTorch expressions of the reference
    def _decode(self, q, k, v, gt, st):
        if ops.native_on(q) and q.shape[-1] == 128:
            last = st.get("last_hidden_state")
            if last is None or last.dtype != torch.float32 or not last.is_contiguous():
                B, _, H, D = q.shape
                last = (last.float().contiguous() if last is not None
                        else torch.zeros(B, H, D, D, dtype=torch.float32, device=q.device))
            o = ops.retention_decode(q, k, v, gt, last)
            st["last_hidden_state"] = last
            return o
        qh, kh, vh = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
        o, st["last_hidden_state"] = ops.ref.recurrent_gate_retention(qh, kh, vh, gt.transpose(1, 2),
                                                                       st.get("last_hidden_state"))
        return o.transpose(1, 2)

    def _prefill(self, q, k, v, gt, st):
        index_mask = st.get("index_mask")
        last = st.get("last_hidden_state")
        if ops.native_on(q) and q.shape[-1] == 128:
            o, st["last_hidden_state"] = ops.retention_prefill(q, k, v, gt, last, index_mask)
            return o
        qh, kh, vh, gh = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), gt.transpose(1, 2)
        st["last_hidden_state"] = ops.ref.retention_prefill_state(kh, vh, gh, index_mask, last)
        L = qh.shape[2]
        cs = self.args.chunk_size
        if L % cs == 0:
            o = ops.ref.chunk_gate_retention(qh, kh, vh, gh, chunk_size=cs, last_hidden_state=last)
        else:
            o = ops.ref.parallel_gate_retention(qh, kh, vh, gh)
            if last is not None:
                G = gh.float().cumsum(-1)
                o = o + (qh * G[..., None].exp().to(qh.dtype)) @ last
        return o.transpose(1, 2)


class SlidingWindowAttention(nn.Module):
    """Causal attention over the last ``window`` keys (yoco/models/decoder/sliding_window_attention.py:15-69)."""

    def __init__(self, args):
        super().__init__()
        self.args = args
        self.embed_dim = args.dim
        self.num_heads = args.n_self_heads // args.model_parallel_size
        self.window_size = args.sliding_window
        self.head_dim = args.dim // args.n_self_heads
        d = args.dim
        self.qkv_proj = MergedLinear(d, [d, d, d], ["q_proj", "k_proj", "v_proj"], [I.init_method] * 3)
        self.out_proj = Linear(d, d, I.init_method, parallel="row")

    def forward(self, x, rel_pos, start_pos=0, incremental_state=None, residual=None):
        B, L, _ = x.shape
        H, D = self.num_heads, self.head_dim
        d = H * D
        y = self.qkv_proj(TP.copy_to_tp(x))
        q = ops.rope(y[..., :d].view(B, L, H, D), *rel_pos)
        k = ops.rope(y[..., d:2 * d].view(B, L, H, D), *rel_pos)
        v = y[..., 2 * d:].view(B, L, H, D)
        if incremental_state is not None:
            st = incremental_state
            w = self.window_size
            if "prev_key" not in st:
                st["prev_key"] = torch.empty(max(self.args.max_batch_size, B), w, H, D, device=x.device, dtype=x.dtype)
                st["prev_value"] = torch.empty_like(st["prev_key"])
                st["filled"] = 0
            filled = st["filled"]
            key = torch.cat([st["prev_key"][:B, :filled], k], dim=1)
            value = torch.cat([st["prev_value"][:B, :filled], v], dim=1)
            keep = min(w, key.shape[1])
            st["prev_key"][:B, :keep] = key[:, -keep:]
            st["prev_value"][:B, :keep] = value[:, -keep:]
            st["filled"] = keep
            o = ops.ref.attention(q, key, value, causal=True, window=w, q_offset=key.shape[1] - L)
        elif CP.cp_size() > 1:
            kk, vv = CP.gather_seq(k, 1), CP.gather_seq(v, 1)
            o = ops.ref.attention(q, kk, vv, causal=True, window=self.window_size, q_offset=CP.cp_rank() * L)
        else:
            o = ops.attention(q, k, v, causal=True, window=self.window_size)
        return self.out_proj(o.reshape(B, L, H * D), residual)


class CrossAttention(nn.Module):
    """q_proj + RoPE, causal GQA attention on the shared K/V, out_proj (yoco/models/decoder/cross_attention.py)."""

    def __init__(self, args):
        super().__init__()
        self.args = args
        self.embed_dim = args.dim
        self.num_heads = args.n_attn_heads // args.model_parallel_size
        self.num_kv_heads = args.n_attn_kv_heads // args.model_parallel_size
        self.head_dim = args.dim // args.n_attn_heads
        self.q_proj = Linear(args.dim, args.dim, I.init_method, parallel="column")
        self.out_proj = Linear(args.dim, args.dim, I.init_method, parallel="row")

    def forward(self, x, key, value, rel_pos, residual=None, q_offset: Optional[int] = None):
        B, L, _ = x.shape
        q = ops.rope(self.q_proj(TP.copy_to_tp(x)).view(B, L, self.num_heads, self.head_dim), *rel_pos)
        if q_offset is None and CP.cp_size() > 1 and key.shape[1] == CP.cp_size() * L:
            q_offset = CP.cp_rank() * L              # this rank's block inside the gathered sequence
        if key.shape[1] != L:
            off = key.shape[1] - L if q_offset is None else q_offset
            o = ops.ref.attention(q, key, value, causal=True, q_offset=off)
        else:
            o = ops.attention(q, key, value, causal=True)
        return self.out_proj(o.reshape(B, L, self.num_heads * self.head_dim), residual)
