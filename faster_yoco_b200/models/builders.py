"""Model builders behind ``--arch`` (yoco/models/yoco.py:75-158, yoco/models/transformer.py:65-138).

``build_yoco(cfg, vocab_size)``: from a registered architecture preset (``yoco_3b`` ...) plus CLI overrides, or --
with ``yoco_model`` -- from ``<yoco_model>/params.json``; in both cases ``max_batch_size`` / ``max_seq_len`` come
from the batch size and ``tokens_per_sample``. ``load_ckpt`` loads a state dict with the reference's parameter
names (a bare dict or a full checkpoint, ``decoder.model.`` prefix or not). ``--sliding-window N`` is forwarded into
the model arguments (the reference's ``LanguageConfig.sliding_window`` never reached ``YOCOArgs``).
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Optional

import torch

from ..config import YOCOArgs, build_args
from ..registry import register_model


@dataclass
class ModelConfig:
    arch: str = "yoco_3b"
    dim: Optional[int] = None
    hidden_dim: Optional[int] = None
    n_layers: Optional[int] = None
    n_self_heads: Optional[int] = None
    n_attn_heads: Optional[int] = None
    n_attn_kv_heads: Optional[int] = None
    n_heads: Optional[int] = None                  # LLaMA
    n_kv_heads: Optional[int] = None               # LLaMA
    batch_size: int = 1
    tokens_per_sample: int = 2048
    share_input_output_embed: bool = False
    sliding_window: Optional[int] = None
    rope_theta: Optional[float] = None
    checkpoint_activations: bool = False
    yoco_model: Optional[str] = None
    llama_model: Optional[str] = None
    load_ckpt: Optional[str] = None
    model_parallel_size: int = 1
    init_std: Optional[float] = None


def yoco_args(cfg: ModelConfig, vocab_size: int) -> YOCOArgs:
    if cfg.yoco_model is not None:
        args = YOCOArgs.from_json_file(os.path.join(cfg.yoco_model, "params.json"))
    else:
        args = build_args(cfg.arch, dim=cfg.dim, hidden_dim=cfg.hidden_dim, n_layers=cfg.n_layers,
                          n_self_heads=cfg.n_self_heads, n_attn_heads=cfg.n_attn_heads,
                          n_attn_kv_heads=cfg.n_attn_kv_heads, vocab_size=vocab_size, rope_theta=cfg.rope_theta,
                          share_input_output_embed=cfg.share_input_output_embed)
    args.max_batch_size = cfg.batch_size
    args.max_seq_len = cfg.tokens_per_sample
    args.model_parallel_size = cfg.model_parallel_size
    args.load_checkpoint = cfg.load_ckpt is not None
    args.checkpoint_activations = cfg.checkpoint_activations
    if cfg.sliding_window:
        args.sliding_window = int(cfg.sliding_window)
    if cfg.init_std is not None:
        args.init_std = cfg.init_std
    return args


@register_model("yoco")
def build_yoco(cfg: ModelConfig, vocab_size: int, device=None, dtype=None):
    from .yoco import YOCO
    from ..train.checkpoint import load_model_weights
    from ..parallel import tp as TP
    args = yoco_args(cfg, vocab_size)
    with torch.device(device or "cpu"):
        model = YOCO(args)
    if dtype is not None:
        model = model.to(dtype)
    if cfg.load_ckpt is not None:
        if TP.tp_size() > 1:                       # a full (TP = 1) checkpoint, sliced for this rank
            from .yoco import shard_state_dict
            from ..train.checkpoint import PREFIX
            ck = torch.load(cfg.load_ckpt, map_location="cpu", mmap=True)
            sd = ck.get("model", ck)
            sd = {(k[len(PREFIX):] if k.startswith(PREFIX) else k): v for k, v in sd.items()}
            model.load_state_dict(shard_state_dict(sd, TP.tp_size(), TP.tp_rank()))
        else:
            load_model_weights(model, cfg.load_ckpt)
    return model


@register_model("llama")
def build_llama_model(cfg: ModelConfig, vocab_size: int, device=None, dtype=None):
    from .transformer import build_llama
    arch = cfg.arch if cfg.arch.startswith("llama") else "llama_from_scratch"
    over = {k: getattr(cfg, k) for k in ("dim", "n_layers", "n_heads", "n_kv_heads", "rope_theta", "sliding_window")
            if getattr(cfg, k) is not None}
    with torch.device(device or "cpu"):
        m = build_llama(arch, vocab_size, batch_size=cfg.batch_size, tokens_per_sample=cfg.tokens_per_sample,
                        llama_model=cfg.llama_model, load_ckpt=cfg.load_ckpt,
                        checkpoint_activations=cfg.checkpoint_activations,
                        model_parallel_size=cfg.model_parallel_size, **over)
    if dtype is not None:
        m = m.to(dtype)
    return m


def model_family(arch: str) -> str:
    return "llama" if arch.startswith("llama") else "yoco"
