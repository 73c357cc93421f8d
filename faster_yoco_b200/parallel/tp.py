"""Megatron-style tensor parallelism (the ``fairseq.model_parallel.megatron.mpu`` API the reference's layers are
declared with: yoco/models/decoder/gate_retention.py:40-46, feedforward_network.py:24-26, decoder/transformer.py:66-69,
decoder/yoco.py:205-206,274-276; TP-sharded checkpoint load decoder/transformer.py:239-251).

* ``init_model_parallel(tp)`` splits the world into TP groups of ``tp`` consecutive ranks (and the matching
  data-parallel groups of ranks with equal TP rank).
* ``ColumnParallelLinear``: weight rows (output features) split across the TP group; the input enters through
  ``copy_to_tp`` (identity forward, all-reduce of the input gradient), the output is optionally all-gathered.
* ``RowParallelLinear``: weight columns (input features) split; partial products all-reduced (``reduce_from_tp``).
* ``VocabParallelEmbedding``: vocabulary rows split; ids outside this rank's range contribute zeros; all-reduce.

Every parallel layer initialises the FULL master weight with the given init function (same RNG stream on every TP
rank) and keeps its slice, so a TP run starts from exactly the weights of the TP=1 run. Local products use
``ops.linear`` (the tcgen05 GEMM on B200). With TP size 1 every collective is the identity.
"""
from __future__ import annotations

from typing import Callable, List, Optional

import torch
import torch.distributed as dist
import torch.nn as nn

from .. import ops

_TP_GROUP = None
_DP_GROUP = None
_TP_SIZE = 1
_TP_RANK = 0


def init_model_parallel(tp_size: int):
    """Collective over the default group. Returns (tp_group, dp_group)."""
    global _TP_GROUP, _DP_GROUP, _TP_SIZE, _TP_RANK
    world = dist.get_world_size() if dist.is_initialized() else 1
    rank = dist.get_rank() if dist.is_initialized() else 0
    if world % tp_size:
        raise ValueError(f"world size {world} is not divisible by tensor-parallel size {tp_size}")
    _TP_SIZE, _TP_RANK = tp_size, rank % tp_size
    if not dist.is_initialized() or world == 1:
        return None, None
    for start in range(0, world, tp_size):
        g = dist.new_group(list(range(start, start + tp_size)))
        if start <= rank < start + tp_size:
            _TP_GROUP = g
    for r in range(tp_size):
        g = dist.new_group(list(range(r, world, tp_size)))
        if rank % tp_size == r:
            _DP_GROUP = g
    return _TP_GROUP, _DP_GROUP


def destroy_model_parallel():
    global _TP_GROUP, _DP_GROUP, _TP_SIZE, _TP_RANK
    _TP_GROUP = _DP_GROUP = None
    _TP_SIZE, _TP_RANK = 1, 0


def tp_size() -> int:
    return _TP_SIZE


def tp_rank() -> int:
    return _TP_RANK


def tp_group():
    return _TP_GROUP


def dp_group():
    return _DP_GROUP


def model_parallel_is_initialized() -> bool:
    return _TP_GROUP is not None or _TP_SIZE == 1


# ----------------------------------------------------------------------------------------------------------------------
# region functions


def _all_reduce(x: torch.Tensor) -> torch.Tensor:
    if _TP_SIZE == 1:
        return x
    x = x.contiguous()
    dist.all_reduce(x, group=_TP_GROUP)
    return x


def _gather_last(x: torch.Tensor) -> torch.Tensor:
    if _TP_SIZE == 1:
        return x
    parts = [torch.empty_like(x) for _ in range(_TP_SIZE)]
    dist.all_gather(parts, x.contiguous(), group=_TP_GROUP)
    return torch.cat(parts, dim=-1)


def _split_last(x: torch.Tensor) -> torch.Tensor:
    if _TP_SIZE == 1:
        return x
    n = x.shape[-1] // _TP_SIZE
    return x[..., _TP_RANK * n:(_TP_RANK + 1) * n].contiguous()


class _CopyToTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        return x

    @staticmethod
    def backward(ctx, g):
        return _all_reduce(g.clone())


class _ReduceFromTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        return _all_reduce(x.clone())

    @staticmethod
    def backward(ctx, g):
        return g


class _GatherFromTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        return _gather_last(x)

    @staticmethod
    def backward(ctx, g):
        return _split_last(g)


class _ScatterToTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        return _split_last(x)

    @staticmethod
    def backward(ctx, g):
        return _gather_last(g)


def copy_to_tp(x):
    return x if _TP_SIZE == 1 else _CopyToTP.apply(x)


def reduce_from_tp(x):
    return x if _TP_SIZE == 1 else _ReduceFromTP.apply(x)


def gather_from_tp(x):
    return x if _TP_SIZE == 1 else _GatherFromTP.apply(x)


def scatter_to_tp(x):
    return x if _TP_SIZE == 1 else _ScatterToTP.apply(x)


# reference names (fairseq mpu)
copy_to_model_parallel_region = copy_to_tp
reduce_from_model_parallel_region = reduce_from_tp
gather_from_model_parallel_region = gather_from_tp
scatter_to_model_parallel_region = scatter_to_tp


# ----------------------------------------------------------------------------------------------------------------------
# layers


def mark_sharded(p: torch.nn.Parameter) -> torch.nn.Parameter:
    """Tag a parameter that holds only this rank's slice of the logical weight (the ZeRO trainer counts replicated
    parameters once, sharded ones once per TP rank, in the global gradient norm)."""
    if _TP_SIZE > 1:
        p._fyb_tp_sharded = True
    return p


def is_sharded(p: torch.Tensor) -> bool:
    return bool(getattr(p, "_fyb_tp_sharded", False))


def _master_slice(shape, init: Optional[Callable], dim: int, dtype=None, device=None) -> torch.Tensor:
    full = torch.empty(shape, dtype=dtype or torch.float32, device=device)
    if init is not None:
        init(full)
    n = shape[dim] // _TP_SIZE
    return full.narrow(dim, _TP_RANK * n, n).clone()


class ColumnParallelLinear(nn.Module):
    def __init__(self, in_features: int, out_features: int, bias: bool = False, gather_output: bool = True,
                 init_method: Optional[Callable] = None):
        super().__init__()
        if out_features % _TP_SIZE:
            raise ValueError(f"out_features {out_features} not divisible by TP size {_TP_SIZE}")
        if bias:
            raise ValueError("bias is not supported (no layer of the model family uses one)")
        self.in_features, self.out_features, self.gather_output = in_features, out_features, gather_output
        self.init_method = init_method
        self.weight = mark_sharded(nn.Parameter(_master_slice((out_features, in_features), init_method, 0)))

    @torch.no_grad()
    def reset_parameters(self, init_override=None):
        fn = init_override or self.init_method
        if fn is not None:
            self.weight.copy_(_master_slice((self.out_features, self.in_features), fn, 0))

    def forward(self, x):
        y = ops.linear(copy_to_tp(x), self.weight)
        return gather_from_tp(y) if self.gather_output else y


class RowParallelLinear(nn.Module):
    def __init__(self, in_features: int, out_features: int, bias: bool = False, input_is_parallel: bool = False,
                 init_method: Optional[Callable] = None):
        super().__init__()
        if in_features % _TP_SIZE:
            raise ValueError(f"in_features {in_features} not divisible by TP size {_TP_SIZE}")
        if bias:
            raise ValueError("bias is not supported (no layer of the model family uses one)")
        self.in_features, self.out_features, self.input_is_parallel = in_features, out_features, input_is_parallel
        self.init_method = init_method
        self.weight = mark_sharded(nn.Parameter(_master_slice((out_features, in_features), init_method, 1)))

    @torch.no_grad()
    def reset_parameters(self, init_override=None):
        fn = init_override or self.init_method
        if fn is not None:
            self.weight.copy_(_master_slice((self.out_features, self.in_features), fn, 1))

    def forward(self, x, residual=None):
        if not self.input_is_parallel:
            x = scatter_to_tp(x)
        y = reduce_from_tp(ops.linear(x, self.weight))
        return y + residual if residual is not None else y


class VocabParallelEmbedding(nn.Module):
    def __init__(self, num_embeddings: int, embedding_dim: int, padding_idx: int = -1,
                 init_method: Optional[Callable] = None):
        super().__init__()
        if num_embeddings % _TP_SIZE:
            raise ValueError(f"vocabulary {num_embeddings} not divisible by TP size {_TP_SIZE}")
        self.num_embeddings, self.embedding_dim = num_embeddings, embedding_dim
        self.per = num_embeddings // _TP_SIZE
        self.start = _TP_RANK * self.per
        self.init_method = init_method
        self.weight = mark_sharded(nn.Parameter(_master_slice((num_embeddings, embedding_dim), init_method, 0)))

    @torch.no_grad()
    def reset_parameters(self, init_override=None):
        fn = init_override or self.init_method
        if fn is not None:
            self.weight.copy_(_master_slice((self.num_embeddings, self.embedding_dim), fn, 0))

    def forward(self, ids: torch.Tensor, scale: float = 1.0):
        if _TP_SIZE == 1:
            return ops.embedding(ids, self.weight, scale)
        outside = (ids < self.start) | (ids >= self.start + self.per)
        local = torch.where(outside, torch.zeros_like(ids), ids - self.start)
        out = nn.functional.embedding(local, self.weight) * scale
        out = out.masked_fill(outside[..., None], 0)
        return reduce_from_tp(out)


def shard_for_rank(name: str, t: torch.Tensor, vocab_rows: List[str], column: List[str], row: List[str],
                   size: int, rank: int) -> torch.Tensor:
    """Slice a full (TP=1) tensor for TP rank `rank` by the name rules of a model: vocabulary / column-parallel
    weights split along dim 0, row-parallel along dim 1, everything else replicated."""
    if size == 1:
        return t
    if any(k in name for k in vocab_rows) or any(k in name for k in column):
        n = t.shape[0] // size
        return t[rank * n:(rank + 1) * n]
    if any(k in name for k in row):
        n = t.shape[1] // size
        return t[:, rank * n:(rank + 1) * n]
    return t
