"""Context (sequence) parallelism for YOCO training: the tokens of each sequence are split into equal contiguous
blocks, one per rank of a context-parallel group. YOCO needs very little exchange for this (the reference has no
distributed sequence parallelism; this follows its long-context design, gate_recurrent.py:230-251, and the shared
KV cache, decoder/yoco.py:240-247):

* gated retention is a linear recurrence: each rank runs its block with a zero initial state and publishes its
  block's final state ``S = sum_j k_j^T v_j exp(G_end - G_j)`` (one [H, D, D] fp32 matrix per layer) and total
  decay ``exp(G_end)``; the state entering block r is the decayed prefix sum of the earlier blocks' states, and
  adds ``(q exp(G)) @ S_in`` to the block's output;
* the cross-decoder's single shared K / V is gathered along the sequence once per forward (all cross layers reuse
  it), and each rank's queries attend causally with their absolute offset;
* sliding-window attention gathers K / V the same way (a rank needs only the previous window, the gather keeps the
  code simple).

Gradients of the parameters are per-rank partial sums, so the ZeRO trainer's data-parallel gradient sum over all
ranks yields the full-sequence gradient unchanged; only the gathers need the custom backward below (all-reduce of
the gathered gradient, then this rank's slice -- gloo has no reduce-scatter).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

_CP_GROUP = None
_CP_SIZE = 1
_CP_RANK = 0


def init_context_parallel(cp_size: int):
    """Collective over the default group: context-parallel groups of `cp_size` consecutive ranks."""
    global _CP_GROUP, _CP_SIZE, _CP_RANK
    world = dist.get_world_size() if dist.is_initialized() else 1
    rank = dist.get_rank() if dist.is_initialized() else 0
    if world % cp_size:
        raise ValueError(f"world size {world} is not divisible by context-parallel size {cp_size}")
    _CP_SIZE, _CP_RANK = cp_size, rank % cp_size
    if cp_size == 1 or not dist.is_initialized():
        return None
    for start in range(0, world, cp_size):
        g = dist.new_group(list(range(start, start + cp_size)))
        if start <= rank < start + cp_size:
            _CP_GROUP = g
    return _CP_GROUP


def destroy_context_parallel():
    global _CP_GROUP, _CP_SIZE, _CP_RANK
    _CP_GROUP, _CP_SIZE, _CP_RANK = None, 1, 0


def cp_size() -> int:
    return _CP_SIZE


def cp_rank() -> int:
    return _CP_RANK


def cp_group():
    return _CP_GROUP


class _GatherSeq(torch.autograd.Function):
    """all_gather along `dim` within the context-parallel group; backward = all-reduce + own slice."""

    @staticmethod
    def forward(ctx, x, dim):
        ctx.dim, ctx.n = dim, x.shape[dim]
        parts = [torch.empty_like(x) for _ in range(_CP_SIZE)]
        dist.all_gather(parts, x.contiguous(), group=_CP_GROUP)
        return torch.cat(parts, dim)

    @staticmethod
    def backward(ctx, g):
        g = g.contiguous().clone()
        dist.all_reduce(g, group=_CP_GROUP)
        return g.narrow(ctx.dim, _CP_RANK * ctx.n, ctx.n), None


def gather_seq(x: torch.Tensor, dim: int = 1) -> torch.Tensor:
    return x if _CP_SIZE == 1 else _GatherSeq.apply(x, dim)


def gather_stack(x: torch.Tensor) -> torch.Tensor:
    """[cp, *x.shape]: every rank's tensor, with the same autograd rule."""
    return gather_seq(x.unsqueeze(0), 0)


def retention_carry(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor) -> torch.Tensor:
    """Cross-block term of gated retention under context parallelism. q, k, v: [B, H, L, D] (this rank's block,
    k unscaled), g: [B, H, L] per-step log decays. Returns (q exp(G)) @ S_in, [B, H, L, Dv] (fp32)."""
    if _CP_SIZE == 1:
        return torch.zeros(*q.shape[:-1], v.shape[-1], dtype=torch.float32, device=q.device)
    D = k.shape[-1]
    G = g.float().cumsum(-1)                                              # [B, H, L]
    g_end = G[..., -1:]
    w = (g_end - G).exp().unsqueeze(-1)                                   # decay of each key to the block end
    S_loc = (k.float() * D ** -0.5).transpose(-1, -2) @ (v.float() * w)   # [B, H, D, Dv]
    dec = g_end.squeeze(-1).exp()                                         # [B, H]
    S_all = gather_stack(S_loc)                                           # [cp, B, H, D, Dv]
    d_all = gather_stack(dec)                                             # [cp, B, H]
    S_in = torch.zeros_like(S_loc)
    for r in range(_CP_RANK):                                             # state entering this block
        S_in = S_in * d_all[r][..., None, None] + S_all[r]
    # every rank must run the gathers' backward (a collective) even where it uses none of their outputs (rank 0):
    # a zero-weighted term keeps them in the graph, so all ranks issue the same collectives in the same order
    tie = 0.0 * (S_all.sum() + d_all.sum())
    return (q.float() * G.exp().unsqueeze(-1)) @ S_in + tie
