"""Shared set-up of the train / validate entry points: process group, device, task, model."""
from __future__ import annotations

import numpy as np
import torch

from .. import ops
from ..models.builders import ModelConfig, model_family
from ..parallel import dist as D
from ..registry import get_model, get_task
from ..tasks.base import TaskConfig


def setup_runtime(args):
    dev_index = D.init(timeout_s=600)
    use_cuda = torch.cuda.is_available() and not args.cpu
    device = torch.device("cuda", dev_index) if use_cuda else torch.device("cpu")
    ops.set_backend(args.kernels if use_cuda else "torch")
    np.random.seed(args.seed)
    torch.manual_seed(args.seed)
    if args.fp16:
        raise SystemExit("--fp16 is not supported: this framework trains in bf16 (as the reference recipe)")
    if args.model_parallel_size > 1:
        from ..parallel import tp
        tp.init_model_parallel(args.model_parallel_size)
    if getattr(args, "context_parallel_size", 1) > 1:
        if args.model_parallel_size > 1:
            raise SystemExit("context and tensor parallelism together are not supported")
        from ..parallel import context
        context.init_context_parallel(args.context_parallel_size)
    return device


def task_config(args) -> TaskConfig:
    return TaskConfig(data=getattr(args, "data", None), tokens_per_sample=args.tokens_per_sample,
                      max_target_positions=args.max_target_positions, llama_model=args.llama_model,
                      tiktoken_model=args.tiktoken_model, batch_read_ahead=args.batch_read_ahead,
                      pad_to_max_len=args.pad_to_max_len, absolute_path=args.absolute_path,
                      tokenizer_pad_to_multiple=args.tokenizer_pad_to_multiple, seed=args.seed,
                      batch_size=args.batch_size, data_dir=args.data_dir, eval_data=args.eval_data)


def build_task(args):
    return get_task(args.task).setup_task(task_config(args))


def build_model(args, task, device):
    cfg = ModelConfig(arch=args.arch, dim=args.dim, hidden_dim=args.hidden_dim, n_layers=args.n_layers,
                      n_self_heads=args.n_self_heads, n_attn_heads=args.n_attn_heads,
                      n_attn_kv_heads=args.n_attn_kv_heads, n_heads=args.n_heads, n_kv_heads=args.n_kv_heads,
                      batch_size=args.batch_size, tokens_per_sample=args.tokens_per_sample,
                      share_input_output_embed=args.share_input_output_embed, sliding_window=args.sliding_window,
                      rope_theta=args.rope_theta, checkpoint_activations=args.checkpoint_activations,
                      yoco_model=args.yoco_model, llama_model=args.llama_model, load_ckpt=args.load_ckpt,
                      model_parallel_size=args.model_parallel_size, init_std=args.init_std)
    dtype = torch.bfloat16 if (args.bf16 or device.type == "cuda") else torch.float32
    family = model_family(args.arch)
    return get_model(family)(cfg, task.tokenizer.n_words, device=device, dtype=dtype), family
