"""LLaMA-style baseline decoder (yoco/models/decoder/transformer.py:34-251, yoco/models/transformer.py:65-138).

GQA attention with NeoX (half-split) RoPE at angles ``t / theta ** (arange(0, D, 2) / D)``, optional sliding window,
KV cache for incremental decoding; SwiGLU FFN ``w2(silu(w1 x) * w3 x)`` of width ``int(8 dim / 3)``; pre-norm RMSNorm
blocks; untied output projection returning fp32 logits. Layers are declared tensor-parallel (``parallel/tp.py``);
``load_state_dict`` slices a full checkpoint for this TP rank like the reference. Matmuls run on ``ops.linear``
(tcgen05 GEMM where the shape is 16-byte aligned), attention on ``ops.attention`` (sm_100a kernel for head dim 128).
"""
from __future__ import annotations

import dataclasses
import json
import os
from dataclasses import dataclass
from typing import Optional, Tuple

import torch
import torch.nn as nn

from .. import ops
from ..parallel import tp as TP
from . import init as I
from .layers import RMSNorm


@dataclass
class LlamaArgs:
    dim: int
    n_layers: int
    head_dim: int
    hidden_dim: int
    n_heads: int
    n_kv_heads: int
    norm_eps: float
    vocab_size: int
    max_batch_size: int = 0
    max_seq_len: int = -1
    model_parallel_size: int = 1
    load_checkpoint: bool = False
    rope_theta: float = 10000.0
    sliding_window: Optional[int] = None

    @classmethod
    def from_json_file(cls, path: str, **overrides) -> "LlamaArgs":
        with open(path) as f:
            params = json.load(f)
        params.update({k: v for k, v in overrides.items() if v is not None})
        known = {f.name for f in dataclasses.fields(cls)}
        return cls(**{k: v for k, v in params.items() if k in known})


class Attention(nn.Module):
    def __init__(self, args: LlamaArgs):
        super().__init__()
        self.args = args
        self.head_dim = args.head_dim
        self.n_heads = args.n_heads // args.model_parallel_size
        self.n_kv_heads = args.n_kv_heads // args.model_parallel_size
        self.window = args.sliding_window
        self.cache_len = args.sliding_window - 1 if args.sliding_window is not None else args.max_seq_len
        hd, kvd = args.n_heads * args.head_dim, args.n_kv_heads * args.head_dim
        self.wq = TP.ColumnParallelLinear(args.dim, hd, gather_output=False, init_method=I.init_method)
        self.wk = TP.ColumnParallelLinear(args.dim, kvd, gather_output=False, init_method=I.init_method)
        self.wv = TP.ColumnParallelLinear(args.dim, kvd, gather_output=False, init_method=I.init_method)
        self.wo = TP.RowParallelLinear(hd, args.dim, input_is_parallel=True, init_method=I.init_method)

    def forward(self, x, rel_pos, start_pos: int, incremental_state=None, residual=None):
        B, L, _ = x.shape
        q = self.wq(x).view(B, L, self.n_heads, self.head_dim)
        k = self.wk(x).view(B, L, self.n_kv_heads, self.head_dim)
        v = self.wv(x).view(B, L, self.n_kv_heads, self.head_dim)
        q = ops.rope(q, *rel_pos, interleaved=False)
        k = ops.rope(k, *rel_pos, interleaved=False)
        if incremental_state is None:
            o = ops.attention(q, k, v, causal=True, window=self.window)
        else:
            st = incremental_state
            if self.window is None:
                need = start_pos + L
                have = st["cache_k"].shape[1] if "cache_k" in st else 0
                if need > have:             # max_seq_len positions, grown for longer prompts + generation
                    size = max(self.cache_len, (need + 1023) // 1024 * 1024)
                    shape = (max(self.args.max_batch_size, B), size, self.n_kv_heads, self.head_dim)
                    nk = torch.zeros(shape, dtype=k.dtype, device=k.device)
                    nv = torch.zeros(shape, dtype=v.dtype, device=v.device)
                    if have:
                        nk[:, :have] = st["cache_k"]
                        nv[:, :have] = st["cache_v"]
                    st["cache_k"], st["cache_v"] = nk, nv
                st["cache_k"][:B, start_pos:start_pos + L] = k
                st["cache_v"][:B, start_pos:start_pos + L] = v
                key = st["cache_k"][:B, :start_pos + L]
                value = st["cache_v"][:B, :start_pos + L]
            else:
                # the last (window - 1) keys before this block are all a query of the block can still see
                prev_k = st.get("cache_k")
                key = k if prev_k is None else torch.cat([prev_k[:B], k], 1)
                value = v if prev_k is None else torch.cat([st["cache_v"][:B], v], 1)
                keep = min(self.cache_len, key.shape[1])
                st["cache_k"], st["cache_v"] = key[:, -keep:].clone(), value[:, -keep:].clone()
            o = ops.ref.attention(q, key, value, causal=True, window=self.window, q_offset=key.shape[1] - L)
        return self.wo(o.reshape(B, L, self.n_heads * self.head_dim), residual)


class FeedForward(nn.Module):
    def __init__(self, args: LlamaArgs):
        super().__init__()
        self.w1 = TP.ColumnParallelLinear(args.dim, args.hidden_dim, gather_output=False, init_method=I.init_method)
        self.w2 = TP.RowParallelLinear(args.hidden_dim, args.dim, input_is_parallel=True, init_method=I.init_method)
        self.w3 = TP.ColumnParallelLinear(args.dim, args.hidden_dim, gather_output=False, init_method=I.init_method)

    def forward(self, x, residual=None):
        return self.w2(ops.swiglu(self.w1(x), self.w3(x)), residual)


class TransformerBlock(nn.Module):
    def __init__(self, args: LlamaArgs):
        super().__init__()
        self.attention = Attention(args)
        self.feed_forward = FeedForward(args)
        self.attention_norm = RMSNorm(args.dim, eps=args.norm_eps)
        self.ffn_norm = RMSNorm(args.dim, eps=args.norm_eps)

    def forward(self, x, rel_pos, start_pos: int, incremental_state=None):
        h = self.attention(self.attention_norm(x), rel_pos, start_pos, incremental_state, residual=x)
        return self.feed_forward(self.ffn_norm(h), residual=h)


class Transformer(nn.Module):
    COLUMN = ("wq.", "wk.", "wv.", "w1.", "w3.")
    ROW = ("wo.", "w2.")
    VOCAB = ("tok_embeddings", "output")

    def __init__(self, args: LlamaArgs, checkpoint_activations: bool = False):
        super().__init__()
        self.args = args
        self.vocab_size = args.vocab_size
        self.checkpoint_activations = checkpoint_activations
        self.tok_embeddings = TP.VocabParallelEmbedding(args.vocab_size, args.dim, -1, init_method=I.vocab_init_method)
        self.layers = nn.ModuleList([TransformerBlock(args) for _ in range(args.n_layers)])
        self.norm = RMSNorm(args.dim, eps=args.norm_eps)
        self.output = TP.ColumnParallelLinear(args.dim, args.vocab_size, gather_output=False, init_method=None)
        with torch.no_grad():                 # nn.Linear's default init (the reference's output layer is nn.Linear)
            w = torch.empty(args.vocab_size, args.dim)
            nn.init.kaiming_uniform_(w, a=5 ** 0.5)
            n = args.vocab_size // args.model_parallel_size
            self.output.weight.copy_(w[TP.tp_rank() * n:(TP.tp_rank() + 1) * n])
        self._angles = None

    def rel_pos(self, x, start_pos: int):
        need = start_pos + x.size(1)
        if self._angles is None or self._angles.shape[0] < need or self._angles.device != x.device:
            n = max(need, self.args.max_seq_len)
            self._angles = ops.ref.llama_rope_angles(self.args.head_dim, n, self.args.rope_theta, x.device)
        a = self._angles[start_pos:need]
        return torch.cos(a).to(x.dtype), torch.sin(a).to(x.dtype)

    def forward_partial(self, ids, start_pos: int = 0, incremental_state=None):
        h = self.tok_embeddings(ids)
        rel_pos = self.rel_pos(h, start_pos)
        for i, layer in enumerate(self.layers):
            st = None
            if incremental_state is not None:
                st = incremental_state.setdefault(i, {})
            if self.checkpoint_activations and self.training and st is None:
                h = torch.utils.checkpoint.checkpoint(layer, h, rel_pos, start_pos, None, use_reentrant=False)
            else:
                h = layer(h, rel_pos, start_pos, incremental_state=st)
        return self.norm(h)

    def forward(self, ids, start_pos: int = 0, incremental_state=None, return_hidden: bool = False, **unused):
        h = self.forward_partial(ids, start_pos, incremental_state)
        if return_hidden:
            return h, None
        return self.output(h).float(), None

    def output_layer(self, h):
        return self.output(h)

    def load_state_dict(self, state_dict, strict: bool = False, assign: bool = False):
        """Accepts a FULL (TP=1) checkpoint and keeps this rank's slices (decoder/transformer.py:239-251)."""
        size, rank = self.args.model_parallel_size, TP.tp_rank()
        local = {k: TP.shard_for_rank(k, v, list(self.VOCAB), list(self.COLUMN), list(self.ROW), size, rank)
                 for k, v in state_dict.items()}
        return super().load_state_dict(local, strict=strict, assign=assign)


class LLaMA(nn.Module):
    """The task-facing wrapper: negative ids (padding) are mapped to 0 (yoco/models/transformer.py:119-128)."""

    def __init__(self, model: Transformer):
        super().__init__()
        self.model = model

    def forward(self, src_tokens, start_pos: int = 0, **kw):
        src_tokens = torch.where(src_tokens < 0, torch.zeros_like(src_tokens), src_tokens)
        return self.model(src_tokens, start_pos, **kw)

    def max_positions(self):
        return self.model.args.max_seq_len


def llama_args_from_cfg(dim: int, n_layers: int, n_heads: int, n_kv_heads: int, vocab_size: int, *, batch_size: int,
                        tokens_per_sample: int, model_parallel_size: int = 1, rope_theta: float = 10000.0,
                        norm_eps: float = 1e-5, sliding_window: Optional[int] = None,
                        load_checkpoint: bool = False) -> LlamaArgs:
    """From-scratch arguments (yoco/models/transformer.py:76-93): head_dim = dim / heads, hidden = int(8 dim / 3)."""
    return LlamaArgs(dim=dim, n_layers=n_layers, head_dim=dim // n_heads, hidden_dim=int(dim * 8 / 3),
                     n_heads=n_heads, n_kv_heads=n_kv_heads, norm_eps=norm_eps, vocab_size=vocab_size,
                     max_batch_size=batch_size, max_seq_len=tokens_per_sample,
                     model_parallel_size=model_parallel_size, load_checkpoint=load_checkpoint,
                     rope_theta=rope_theta, sliding_window=sliding_window)


LLAMA_ARCHS = {
    # yoco/models/transformer.py:130-138
    "llama_from_scratch": dict(dim=1024, n_layers=8, n_heads=8, n_kv_heads=2, init_from_config=False),
    "llama_from_ckpt": dict(init_from_config=True),
}


def build_llama(arch: str, vocab_size: int, *, batch_size: int, tokens_per_sample: int, llama_model: Optional[str] = None,
                load_ckpt: Optional[str] = None, checkpoint_activations: bool = False, model_parallel_size: int = 1,
                **overrides) -> LLaMA:
    preset = dict(LLAMA_ARCHS[arch])
    preset.update({k: v for k, v in overrides.items() if v is not None})
    if preset.pop("init_from_config"):
        if llama_model is None:
            raise ValueError("llama_from_ckpt needs --llama-model <dir with params.json>")
        args = LlamaArgs.from_json_file(os.path.join(llama_model, "params.json"))
        args.max_batch_size, args.max_seq_len = batch_size, tokens_per_sample
        args.model_parallel_size, args.load_checkpoint = model_parallel_size, load_ckpt is not None
    else:
        args = llama_args_from_cfg(preset["dim"], preset["n_layers"], preset["n_heads"], preset["n_kv_heads"],
                                   vocab_size, batch_size=batch_size, tokens_per_sample=tokens_per_sample,
                                   model_parallel_size=model_parallel_size,
                                   rope_theta=preset.get("rope_theta", 10000.0),
                                   sliding_window=preset.get("sliding_window"), load_checkpoint=load_ckpt is not None)
    model = Transformer(args, checkpoint_activations=checkpoint_activations)
    if load_ckpt is not None:
        model.load_state_dict(torch.load(load_ckpt, map_location="cpu", mmap=True), assign=True)
    return LLaMA(model)
