"""The YOCO decoder-decoder (yoco/models/decoder/yoco.py:51-320).

A self-decoder of ``n_layers // 2`` gated-retention (or sliding-window attention) layers produces the hidden states
from which ONE shared K/V is projected (``kv_layer_norm`` -> ``kv_proj`` -> RoPE on K); ``n_layers // 2``
cross-decoder layers attend to it with causal GQA. Embedding x sqrt(dim) in, final RMSNorm and an untied output
projection out.

Residual adds are folded into the GEMM that produces the mixer / FFN output (``out_proj(o, residual)``), which the
native path executes as the GEMM epilogue.
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import ops
from ..config import YOCOArgs
from ..parallel import context as CP
from ..parallel import tp as TP
from . import init as I
from .layers import (CrossAttention, FeedForwardNetwork, GateRetention, Linear, MergedLinear, RMSNorm,
                     SlidingWindowAttention)


class DecoderLayer(nn.Module):
    """Pre-norm mixer + pre-norm SwiGLU FFN with residuals (yoco/models/decoder/yoco.py:51-125)."""

    def __init__(self, args: YOCOArgs, is_cross_layer: bool = False):
        super().__init__()
        self.args = args
        self.is_cross_layer = is_cross_layer
        if is_cross_layer:
            self.mixer = CrossAttention(args)
        elif args.sliding_window is not None:
            self.mixer = SlidingWindowAttention(args)
        else:
            self.mixer = GateRetention(args)
        self.mixer_layer_norm = RMSNorm(args.dim, eps=args.norm_eps)
        self.ffn = FeedForwardNetwork(args.dim, args.hidden_dim)
        self.final_layer_norm = RMSNorm(args.dim, eps=args.norm_eps)

    def _fused(self, x, key, value, rel_pos):
        """The whole layer as one autograd Function (native training path, see models/fused.py)."""
        from . import fused as Fz
        m, f = self.mixer, self.ffn
        cos, sin = rel_pos
        common = (self.final_layer_norm.weight, f.fc1_gate.weight, f.fc2.weight)
        if self.is_cross_layer:
            cfg = (m.num_heads, m.head_dim, self.args.norm_eps, f.ffn_dim)
            return Fz.CrossLayerFn.apply(x, key, value, self.mixer_layer_norm.weight, m.q_proj.weight,
                                         m.out_proj.weight, *common, cos, sin, cfg)
        if self.args.sliding_window is not None:
            cfg = (m.num_heads, m.head_dim, self.args.norm_eps, m.window_size, f.ffn_dim)
            return Fz.SelfWindowLayerFn.apply(x, self.mixer_layer_norm.weight, m.qkv_proj.weight, m.out_proj.weight,
                                              *common, cos, sin, cfg)
        cfg = (m.num_heads, m.head_dim, self.args.norm_eps, m.subln_eps, m.gate_logit_normalizer, f.ffn_dim)
        return Fz.SelfRetentionLayerFn.apply(x, self.mixer_layer_norm.weight, m.qkvg_proj.weight, m.out_proj.weight,
                                             *common, cos, sin, cfg)

    def forward(self, x, start_pos=0, key=None, value=None, rel_pos=None, incremental_state=None,
                is_prefilling=False):
        from .fused import fused_path_ok
        if incremental_state is None and self.training and fused_path_ok(x, self.mixer.head_dim):
            return self._fused(x, key, value, rel_pos)
        residual = x
        h = self.mixer_layer_norm(x)
        if self.is_cross_layer:
            x = self.mixer(h, key, value, rel_pos=rel_pos, residual=residual)
        elif self.args.sliding_window is not None:
            x = self.mixer(h, rel_pos=rel_pos, start_pos=start_pos, incremental_state=incremental_state,
                           residual=residual)
        else:
            x = self.mixer(h, rel_pos=rel_pos, incremental_state=incremental_state, is_prefilling=is_prefilling,
                           residual=residual)
        residual = x
        h = self.final_layer_norm(x)
        return self.ffn(h, residual=residual)


class _RopeCache:
    """cos/sin tables (model dtype) for positions [start, start+len), built from fp32 angles once per device."""

    def __init__(self, head_dim: int, theta: float, max_len: int):
        self.head_dim, self.theta, self.max_len = head_dim, theta, max_len
        self._angles: Dict = {}
        self._tables: Dict = {}

    def get(self, start: int, length: int, dtype, device):
        key = (start, length, dtype, str(device))
        t = self._tables.get(key)
        if t is None:
            need = max(self.max_len, start + length)
            ang = self._angles.get(str(device))
            if ang is None or ang.shape[0] < need:
                ang = ops.ref.rope_angles(self.head_dim, need, self.theta, device)
                self._angles[str(device)] = ang
            a = ang[start:start + length]
            t = (torch.cos(a).to(dtype), torch.sin(a).to(dtype))
            if len(self._tables) > 64:
                self._tables.clear()
            self._tables[key] = t
        return t


class SelfDecoder(nn.Module):
    def __init__(self, args: YOCOArgs):
        super().__init__()
        self.args = args
        self.layers = nn.ModuleList([DecoderLayer(args, is_cross_layer=False) for _ in range(args.n_layers // 2)])
        self.head_dim = args.dim // args.n_self_heads
        self.block_size = args.chunk_size
        self.rope = _RopeCache(self.head_dim, args.rope_theta, max(args.max_seq_len, 1))
        self.checkpoint_activations = args.checkpoint_activations

    def forward(self, x, incremental_state=None, is_prefilling=False, start_pos=0, comm_hooks=None, bucket0=1):
        pad = 0
        cp = CP.cp_size() > 1 and incremental_state is None
        if is_prefilling and x.size(1) % self.block_size != 0 and self.args.sliding_window is None and not cp:
            pad = self.block_size - x.size(1) % self.block_size
            x = F.pad(x, (0, 0, 0, pad), value=0)
        index_mask = None
        if incremental_state is not None and is_prefilling:
            index_mask = torch.arange(x.size(1), device=x.device) >= (x.size(1) - pad)
        if cp:
            start_pos = start_pos + CP.cp_rank() * x.size(1)      # absolute positions of this rank's block
        rel_pos = self.rope.get(start_pos, x.size(1), x.dtype, x.device)
        for idx, layer in enumerate(self.layers):
            if comm_hooks is not None:
                comm_hooks.before(bucket0 + idx)
                if x.requires_grad:
                    # fires once this layer's backward (all of its weight gradients) is complete
                    x.register_hook(lambda g, b=bucket0 + idx: comm_hooks.ready(b))
            st = None
            if incremental_state is not None:
                st = incremental_state.setdefault(idx, {})
                if is_prefilling:
                    st["index_mask"] = index_mask
            if self.checkpoint_activations and self.training and st is None:
                x = torch.utils.checkpoint.checkpoint(layer, x, start_pos, None, None, rel_pos, None, False,
                                                      use_reentrant=False)
            else:
                x = layer(x, start_pos=start_pos, rel_pos=rel_pos, incremental_state=st, is_prefilling=is_prefilling)
        return x[:, :x.size(1) - pad, :]


class CrossDecoder(nn.Module):
    def __init__(self, args: YOCOArgs):
        super().__init__()
        self.args = args
        self.num_heads = args.n_attn_kv_heads // args.model_parallel_size    # this rank's KV heads
        self.head_dim = args.dim // args.n_attn_heads
        kvd = self.head_dim * args.n_attn_kv_heads
        self.kv_proj = MergedLinear(args.dim, [kvd, kvd], ["k_proj", "v_proj"], [I.init_method, I.init_method])
        self.kv_layer_norm = RMSNorm(args.dim, eps=args.norm_eps)
        self.layers = nn.ModuleList([DecoderLayer(args, is_cross_layer=True) for _ in range(args.n_layers // 2)])
        self.rope = _RopeCache(self.head_dim, args.rope_theta, max(args.max_seq_len, 1))
        self.checkpoint_activations = args.checkpoint_activations

    def shared_kv(self, x, start_pos=0, fused: bool = False):
        B, L, _ = x.shape
        kvd = self.head_dim * self.num_heads
        rel_pos = self.rope.get(start_pos, L, x.dtype, x.device)
        if fused:
            from .fused import SharedKVFn
            key, value = SharedKVFn.apply(x, self.kv_layer_norm.weight, self.kv_proj.weight, *rel_pos,
                                          (self.num_heads, self.head_dim, self.args.norm_eps))
            return key, value, rel_pos
        y = self.kv_proj(TP.copy_to_tp(self.kv_layer_norm(x)))
        key = ops.rope(y[..., :kvd].view(B, L, self.num_heads, self.head_dim), *rel_pos)
        value = y[..., kvd:].view(B, L, self.num_heads, self.head_dim)
        return key, value, rel_pos

    def forward(self, x, incremental_state=None, start_pos=0, skip_cross_decoder=False, comm_hooks=None,
                bucket0=None):
        bsz, seqlen, dim = x.shape
        from .fused import fused_path_ok
        if comm_hooks is not None:
            comm_hooks.before(bucket0)             # shared K/V projection
            if x.requires_grad:
                x.register_hook(lambda g: (comm_hooks.ready(bucket0 + 1), comm_hooks.ready(bucket0)) and None)
        fused = incremental_state is None and self.training and fused_path_ok(x, self.head_dim)
        cp = CP.cp_size() > 1 and incremental_state is None
        if cp:
            start_pos = start_pos + CP.cp_rank() * seqlen
        key, value, rel_pos = self.shared_kv(x, start_pos, fused=fused)
        if cp:                                   # the one shared K / V over the whole sequence, for every layer
            key, value = CP.gather_seq(key, 1), CP.gather_seq(value, 1)
        if incremental_state is not None:
            st = incremental_state
            need = start_pos + seqlen
            have = st["prev_key"].shape[1] if "prev_key" in st else 0
            if need > have:
                # the shared KV cache holds max_seq_len positions; a longer prompt + generation grows it (the
                # filled prefix is kept)
                size = max(self.args.max_seq_len, (need + 1023) // 1024 * 1024)
                shape = (bsz, size, self.num_heads, self.head_dim)
                nk = torch.empty(shape, device=x.device, dtype=x.dtype)
                nv = torch.empty(shape, device=x.device, dtype=x.dtype)
                if have:
                    nk[:, :have] = st["prev_key"]
                    nv[:, :have] = st["prev_value"]
                st["prev_key"], st["prev_value"] = nk, nv
            st["prev_key"][:, start_pos:start_pos + seqlen] = key
            st["prev_value"][:, start_pos:start_pos + seqlen] = value
            key = st["prev_key"][:, :start_pos + seqlen]
            value = st["prev_value"][:, :start_pos + seqlen]
        if skip_cross_decoder:
            return torch.zeros(bsz, 1, dim, device=x.device, dtype=x.dtype)
        for i, layer in enumerate(self.layers):
            if comm_hooks is not None:
                comm_hooks.before(bucket0 + 1 + i)
                if i > 0 and x.requires_grad:
                    x.register_hook(lambda g, b=bucket0 + 1 + i: comm_hooks.ready(b))
            if self.checkpoint_activations and self.training and incremental_state is None:
                x = torch.utils.checkpoint.checkpoint(layer, x, 0, key, value, rel_pos, None, False,
                                                      use_reentrant=False)
            else:
                x = layer(x, key=key, value=value, rel_pos=rel_pos)
        return x


# reference state-dict names of the merged projections: internal param -> (exported names in row-block order)
_MERGED = {
    "mixer.qkvg_proj.weight": ["mixer.q_proj.weight", "mixer.k_proj.weight", "mixer.v_proj.weight",
                               "mixer.g_proj.weight", "mixer.gt_proj.weight"],
    "mixer.qkv_proj.weight": ["mixer.q_proj.weight", "mixer.k_proj.weight", "mixer.v_proj.weight"],
    "ffn.fc1_gate.weight": ["ffn.fc1.weight", "ffn.gate.weight"],
    "kv_proj.weight": ["k_proj.weight", "v_proj.weight"],
}


def _rng_snapshot():
    """CPU generator + the current CUDA device's generator (only when CUDA is already initialised: no new context)."""
    cuda = None
    if torch.cuda.is_available() and torch.cuda.is_initialized():
        cuda = (torch.cuda.current_device(), torch.cuda.get_rng_state())
    return torch.get_rng_state(), cuda


def _rng_restore(snap):
    cpu, cuda = snap
    torch.set_rng_state(cpu)
    if cuda is not None:
        torch.cuda.set_rng_state(cuda[1], cuda[0])


class YOCO(nn.Module):
    def __init__(self, args: YOCOArgs):
        super().__init__()
        self.args = args
        if args.model_parallel_size != TP.tp_size():
            raise ValueError(f"model_parallel_size {args.model_parallel_size} but the tensor-parallel group has "
                             f"{TP.tp_size()} ranks (call parallel.tp.init_model_parallel first)")
        self.embed_scale = math.sqrt(args.dim)
        # the weights come from reset_parameters below, started from this RNG state: what the submodule
        # constructors draw (which differs between the tensor-parallel and single-rank layer classes) does not
        # shift them, so a seed gives the same logical weights at every TP degree
        rng = _rng_snapshot()
        if TP.tp_size() > 1:
            self.embed_tokens = TP.VocabParallelEmbedding(args.vocab_size, args.dim)
            self.output_projection = TP.ColumnParallelLinear(args.dim, args.vocab_size, gather_output=True)
        else:
            self.embed_tokens = nn.Embedding(args.vocab_size, args.dim)
            self.output_projection = Linear(args.dim, args.vocab_size, I.init_method)
        if args.share_input_output_embed:
            self.output_projection.weight = self.embed_tokens.weight
        self.self_decoder = SelfDecoder(args)
        self.cross_decoder = CrossDecoder(args)
        self.layer_norm = RMSNorm(args.dim, eps=args.norm_eps)
        _rng_restore(rng)
        self.reset_parameters()
        self._register_state_dict_hook(YOCO._export_hook)
        self._register_load_state_dict_pre_hook(YOCO._import_hook, with_module=True)

    @torch.no_grad()
    def reset_parameters(self):
        std = self.args.init_std
        override = I.normal_init(std) if std is not None else None
        if isinstance(self.embed_tokens, TP.VocabParallelEmbedding):
            self.embed_tokens.reset_parameters(override or I.vocab_init_method)
            self.output_projection.reset_parameters(override or I.init_method)
        else:
            I.vocab_init_method(self.embed_tokens.weight) if override is None else override(self.embed_tokens.weight)
        for m in self.modules():
            if isinstance(m, (MergedLinear, Linear)):
                m.reset_parameters(override)
            elif isinstance(m, RMSNorm) and m.weight is not None:
                m.weight.fill_(1.0)

    # ------------------------------------------------------------------------------------------------------------
    def param_buckets(self):
        """Parameter groups in forward order (the units of the overlapped gather / reduce): embedding, each
        self-decoder layer, the shared K/V projection, each cross-decoder layer, final norm + output projection."""
        seen = set()

        def grp(params):
            out = []
            for p in params:
                if p.requires_grad and id(p) not in seen:
                    seen.add(id(p))
                    out.append(p)
            return out
        groups = [grp([self.embed_tokens.weight])]
        groups += [grp(l.parameters()) for l in self.self_decoder.layers]
        groups.append(grp(list(self.cross_decoder.kv_proj.parameters()) +
                          list(self.cross_decoder.kv_layer_norm.parameters())))
        groups += [grp(l.parameters()) for l in self.cross_decoder.layers]
        groups.append(grp(list(self.layer_norm.parameters()) + list(self.output_projection.parameters())))
        rest = grp(self.parameters())
        if rest:
            groups[-1] += rest
        return groups

    def forward(self, x, start_pos=0, incremental_state=None, is_prefilling=True, skip_cross_decoder=False,
                return_hidden: bool = False, comm_hooks=None):
        """x: [B, L] token ids -> (logits [B, L, V], None) (yoco/models/decoder/yoco.py:285-315).

        comm_hooks (training with overlapped ZeRO communication): before(b) is called ahead of bucket b's first
        use in forward, ready(b) once its gradients are complete (see param_buckets for the bucket order)."""
        n_self = len(self.self_decoder.layers)
        if comm_hooks is not None:
            comm_hooks.before(0)
        if isinstance(self.embed_tokens, TP.VocabParallelEmbedding):
            h = self.embed_tokens(x, self.embed_scale)
        else:
            h = ops.embedding(x, self.embed_tokens.weight, self.embed_scale)
        h = self.self_decoder(h, incremental_state=incremental_state, is_prefilling=is_prefilling,
                              start_pos=start_pos, comm_hooks=comm_hooks, bucket0=1)
        h = self.cross_decoder(h, start_pos=start_pos, incremental_state=incremental_state,
                               skip_cross_decoder=skip_cross_decoder, comm_hooks=comm_hooks, bucket0=1 + n_self)
        if comm_hooks is not None:
            head = 2 + n_self + len(self.cross_decoder.layers)
            comm_hooks.before(head)
            if h.requires_grad:
                h.register_hook(lambda g: comm_hooks.ready(head))
        h = self.layer_norm(h)
        if return_hidden:
            return h, None
        return self.output_layer(h), None

    def output_layer(self, features):
        return self.output_projection(features)

    # ------------------------------------------------------------------------------------------------------------
    # reference-compatible state dict (split merged projections; drop pad rows)
    @staticmethod
    def _export_hook(module, state_dict, prefix, local_metadata):
        for key in list(state_dict.keys()):
            if not key.startswith(prefix):
                continue
            rel = key[len(prefix):]
            for internal, names in _MERGED.items():
                if rel == internal or rel.endswith("." + internal):
                    base = rel[: len(rel) - len(internal)]
                    mod = module.get_submodule((prefix + base + internal)[len(prefix):].rsplit(".weight", 1)[0])
                    w = state_dict.pop(key)
                    for (off, n), name in zip(mod.offsets(), names):
                        state_dict[prefix + base + name] = w[off:off + n]
                    break
        return state_dict

    @staticmethod
    def _import_hook(module, state_dict, prefix, local_metadata, strict, missing, unexpected, errors):
        for name, mod in module.named_modules():
            if not isinstance(mod, MergedLinear):
                continue
            base = prefix + (name.rsplit(".", 1)[0] + "." if "." in name else "")
            internal_key = prefix + name + ".weight"
            if internal_key in state_dict:
                continue
            leaf = name.rsplit(".", 1)[-1]
            names = [n for n in mod.names]
            keys = [base + n + ".weight" for n in names]
            if all(k in state_dict for k in keys):
                blocks = [state_dict.pop(k) for k in keys]
                w = torch.cat(blocks, 0)
                if w.shape[0] < mod.rows:
                    w = torch.cat([w, w.new_zeros(mod.rows - w.shape[0], w.shape[1])], 0)
                state_dict[internal_key] = w


# reference parameter name suffix -> how a full (TP = 1) tensor is cut for one tensor-parallel rank
_TP_COLUMN = ("mixer.q_proj.weight", "mixer.k_proj.weight", "mixer.v_proj.weight", "mixer.g_proj.weight",
              "mixer.gt_proj.weight", "ffn.fc1.weight", "ffn.gate.weight", "cross_decoder.k_proj.weight",
              "cross_decoder.v_proj.weight", "embed_tokens.weight", "output_projection.weight")
_TP_ROW = ("mixer.out_proj.weight", "ffn.fc2.weight")


def shard_state_dict(full: Dict[str, torch.Tensor], size: int, rank: int) -> Dict[str, torch.Tensor]:
    """This TP rank's slice of a full reference-named state dict (the reference's TP-sliced load,
    yoco/models/decoder/transformer.py:239-251, applied to YOCO's column / row-parallel declarations)."""
    out = {}
    for k, v in full.items():
        if size > 1 and k.endswith(_TP_COLUMN):
            n = v.shape[0] // size
            v = v[rank * n:(rank + 1) * n]
        elif size > 1 and k.endswith(_TP_ROW):
            n = v.shape[1] // size
            v = v[:, rank * n:(rank + 1) * n]
        out[k] = v
    return out


def build_model(args: YOCOArgs, device=None, dtype=None) -> YOCO:
    m = YOCO(args)
    if device is not None or dtype is not None:
        m = m.to(device=device, dtype=dtype)
    return m
