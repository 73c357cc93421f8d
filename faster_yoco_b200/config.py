"""Typed model / training configuration and the architecture registry.

Model hyper-parameters mirror the reference's ``YOCOArgs`` (yoco/models/decoder/yoco.py:33-49) and the fairseq
``LanguageConfig`` dataclass (yoco/models/yoco.py:29-73); the ``yoco_3b`` preset is the reference's only registered
YOCO architecture (yoco/models/yoco.py:146-154). Presets are plain functions that fill unset fields, the way
fairseq's ``register_model_architecture`` presets do, so CLI flags override them.
"""
from __future__ import annotations

import dataclasses
import json
import os
from dataclasses import dataclass, field
from typing import Callable, Dict, Optional


@dataclass
class YOCOArgs:
    """Architecture of one YOCO model (field names and defaults as the reference's YOCOArgs)."""

    dim: int
    n_layers: int
    hidden_dim: int
    n_self_heads: int
    n_attn_heads: int
    n_attn_kv_heads: int
    vocab_size: int
    max_batch_size: int = 0
    max_seq_len: int = -1
    model_parallel_size: int = 1
    load_checkpoint: bool = False
    rope_theta: float = 10000.0
    norm_eps: float = 1e-5
    sliding_window: Optional[int] = None
    # fields below have no counterpart in the reference's YOCOArgs
    init_std: Optional[float] = None       # N(0, init_std) for every weight (benchmarks); None = reference init
    share_input_output_embed: bool = False
    checkpoint_activations: bool = False
    gate_logit_normalizer: int = 16
    chunk_size: int = 256

    @property
    def head_dim(self) -> int:
        return self.dim // self.n_self_heads

    def to_json(self) -> str:
        return json.dumps(dataclasses.asdict(self), indent=2, sort_keys=True)

    @classmethod
    def from_json_file(cls, path: str) -> "YOCOArgs":
        with open(path) as f:
            params = json.load(f)
        known = {f.name for f in dataclasses.fields(cls)}
        return cls(**{k: v for k, v in params.items() if k in known})

    def num_params(self) -> int:
        """Parameter count from the architecture alone (no model instantiation)."""
        d, f, v = self.dim, self.hidden_dim, self.vocab_size
        hd = d // self.n_attn_heads
        kv = hd * self.n_attn_kv_heads
        ffn = 3 * d * f + 2 * d                                    # fc1, gate, fc2 + two layer norms
        if self.sliding_window is None:
            self_mixer = 4 * d * d + self.n_self_heads * d + d * d  # q,k,v,g + gt + out
        else:
            self_mixer = 4 * d * d                                  # q,k,v,out
        cross_mixer = 2 * d * d                                     # q + out
        n_half = self.n_layers // 2
        emb = v * d * (1 if self.share_input_output_embed else 2)
        return emb + n_half * (self_mixer + ffn) + n_half * (cross_mixer + ffn) + 2 * d * kv + d + d


_ARCHS: Dict[str, Callable[[dict], dict]] = {}


def register_arch(name: str):
    def deco(fn):
        _ARCHS[name] = fn
        return fn
    return deco


def arch_names():
    return sorted(_ARCHS)


def _default(a: dict) -> dict:
    a.setdefault("n_attn_kv_heads", a.get("n_attn_heads"))
    a.setdefault("sliding_window", None)
    a.setdefault("rope_theta", 10000.0)
    a.setdefault("share_input_output_embed", False)
    a.setdefault("checkpoint_activations", False)
    return a


@register_arch("yoco_3b")
def yoco_3b(a: dict) -> dict:
    """dim 3072, FFN 8192, 26 layers (13 self + 13 cross), 24 heads, 8 KV heads (reference yoco/models/yoco.py:146-154)."""
    a.setdefault("dim", 3072)
    a.setdefault("hidden_dim", 8192)
    a.setdefault("n_layers", 26)
    a.setdefault("n_self_heads", 24)
    a.setdefault("n_attn_heads", 24)
    a.setdefault("n_attn_kv_heads", 8)
    a.setdefault("vocab_size", 100288)
    return _default(a)


@register_arch("yoco_tiny")
def yoco_tiny(a: dict) -> dict:
    """The CPU/gloo test model: 4 layers, d 256, 4 heads x 64, FFN 688, vocab 1024."""
    a.setdefault("dim", 256)
    a.setdefault("hidden_dim", 688)
    a.setdefault("n_layers", 4)
    a.setdefault("n_self_heads", 4)
    a.setdefault("n_attn_heads", 4)
    a.setdefault("n_attn_kv_heads", 4)
    a.setdefault("vocab_size", 1024)
    return _default(a)


@register_arch("yoco_small")
def yoco_small(a: dict) -> dict:
    """A 1-GPU smoke model with the 3B model's head geometry (head dim 128, GQA 3:1) at small width."""
    a.setdefault("dim", 768)
    a.setdefault("hidden_dim", 2048)
    a.setdefault("n_layers", 4)
    a.setdefault("n_self_heads", 6)
    a.setdefault("n_attn_heads", 6)
    a.setdefault("n_attn_kv_heads", 2)
    a.setdefault("vocab_size", 8192)
    return _default(a)


def build_args(arch: str, **overrides) -> YOCOArgs:
    if arch not in _ARCHS:
        raise KeyError(f"unknown arch {arch!r}; registered: {arch_names()}")
    a = {k: v for k, v in overrides.items() if v is not None}
    a = _ARCHS[arch](a)
    known = {f.name for f in dataclasses.fields(YOCOArgs)}
    return YOCOArgs(**{k: v for k, v in a.items() if k in known})


@dataclass
class OptimConfig:
    """Adam + polynomial-decay schedule (reference recipe scripts/train.sh:11-22)."""

    lr: float = 1.5e-4
    betas: tuple = (0.9, 0.95)
    eps: float = 1e-6
    weight_decay: float = 0.05
    adamw_mode: bool = True           # apex AdamW (decoupled) as fairseq's FusedAdamV2 uses it
    clip_norm: float = 2.0
    warmup_updates: int = 50
    total_num_update: int = 300000
    end_learning_rate: float = 0.0
    power: float = 1.0


@dataclass
class TrainConfig:
    arch: str = "yoco_3b"
    tokens_per_sample: int = 2048
    batch_size: int = 1
    update_freq: int = 1
    max_update: int = 0
    seed: int = 1
    zero_sharding: str = "os"          # none | os: optimizer state sharded (ZeRO-1); gradients go to their owners only
    #                                    (reduce-to-owner, the reference's "ZeRO-2 style" gradient path)
    comm: str = "fused"                # fused (P2P kernels over NVLink) | nccl (the in-repo baseline)
    kernels: str = "native"            # native (sm_100a kernels) | torch (cuBLAS/SDPA baseline)
    layer_graphs: bool = True
    log_interval: int = 10
    save_dir: Optional[str] = None
    save_interval_updates: int = 0
    no_save: bool = True
    data: Optional[str] = None
    bf16: bool = True
    optim: OptimConfig = field(default_factory=OptimConfig)


def env_flag(name: str, default: str = "0") -> bool:
    return os.environ.get(name, default) not in ("0", "", "false", "False")
