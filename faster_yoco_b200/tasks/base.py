"""Task base: tokenizer set-up and the forward / backward step shared by the tasks (the fairseq task contract the
reference's tasks implement: yoco/tasks/gpt.py:58-176, pseudo.py:105-201, harness_eval.py:84-150)."""
from __future__ import annotations

import os
from dataclasses import dataclass, field
from typing import Optional

import torch

from ..data.tokenizers import ByteTokenizer, LLaMATokenizer, TiktokenTokenizer
from ..utils.tracing import phase


@dataclass
class TaskConfig:
    data: Optional[str] = None
    tokens_per_sample: int = 1024
    max_target_positions: Optional[int] = None
    llama_model: Optional[str] = None
    tiktoken_model: Optional[str] = None       # a tiktoken encoding name, a .tiktoken file, or "byte"
    batch_read_ahead: int = 10000
    pad_to_max_len: bool = False
    absolute_path: bool = False
    tokenizer_pad_to_multiple: int = 8
    seed: int = 1
    batch_size: Optional[int] = None
    # harness evaluation
    data_dir: Optional[str] = None
    eval_data: str = ""
    extra: dict = field(default_factory=dict)


def build_task_tokenizer(cfg: TaskConfig):
    """llama_model dir -> its tokenizer.model; tiktoken_model -> tiktoken ("byte" selects the offline byte-level
    tokenizer with the same four special ids); neither -> error, as in the reference."""
    if cfg.llama_model is not None:
        return LLaMATokenizer(os.path.join(cfg.llama_model, "tokenizer.model"))
    if cfg.tiktoken_model is not None:
        if cfg.tiktoken_model == "byte":
            return ByteTokenizer(cfg.tokenizer_pad_to_multiple)
        return TiktokenTokenizer(cfg.tiktoken_model, cfg.tokenizer_pad_to_multiple)
    raise ValueError("No tokenizer model provided (--tiktoken-model / --llama-model)")


class PadDictionary:
    def __init__(self, pad: int):
        self._pad = pad

    def pad(self) -> int:
        return self._pad


class Task:
    def __init__(self, cfg: TaskConfig, tokenizer):
        self.cfg = cfg
        self.tokenizer = tokenizer
        self.datasets = {}

    @classmethod
    def setup_task(cls, cfg: TaskConfig, **kwargs):
        return cls(cfg, build_task_tokenizer(cfg))

    @property
    def target_dictionary(self):
        return PadDictionary(self.tokenizer.pad_id)

    def load_dataset(self, split: str, **kwargs):
        raise NotImplementedError

    def dataset(self, split: str):
        if split not in self.datasets:
            raise KeyError("Dataset not loaded: " + split)
        return self.datasets[split]

    def get_batch_iterator(self, dataset, *, max_sentences=None, seed: int = 1, num_shards: int = 1,
                           shard_id: int = 0, epoch: int = 1, **kwargs):
        raise NotImplementedError

    def train_step(self, sample, model, criterion, optimizer=None, update_num: int = 0, ignore_grad: bool = False):
        """Forward + backward of one sample (the gradient-producing half of an update)."""
        model.train()
        with phase("forward"):
            loss, sample_size, logging_output = criterion(model, sample)
        if ignore_grad:
            loss = loss * 0
        with phase("backward"):
            (optimizer.backward(loss) if optimizer is not None and hasattr(optimizer, "backward")
             else loss.backward())
        return loss, sample_size, logging_output

    def valid_step(self, sample, model, criterion):
        model.eval()
        with torch.no_grad():
            return criterion(model, sample)
