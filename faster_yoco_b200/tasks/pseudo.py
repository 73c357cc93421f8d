"""Pseudo task: endless batches of random token ids for harnesses that need no data (yoco/tasks/pseudo.py:14-201).

As in the reference, ids are drawn from [0, 9999) with the global torch RNG, the target IS the source (no shift) and
``ntokens = batch * length``; the iterator has no state to checkpoint."""
from __future__ import annotations

import torch

from ..registry import register_task
from .base import Task


class PseudoIterator:
    def __init__(self, batch_size: int, length: int, vocab_size: int = 10000):
        self.batch_size, self.length, self.vocab_size = batch_size, length, vocab_size

    def __iter__(self):
        return self

    def __next__(self):
        ids = torch.randint(size=(self.batch_size, self.length), dtype=torch.long, low=0, high=self.vocab_size - 1)
        return {"net_input": {"src_tokens": ids}, "src_tokens": ids, "target": ids,
                "ntokens": self.batch_size * self.length, "nsentences": self.batch_size}

    def __len__(self):
        return 819200000

    def next_epoch_itr(self, **kwargs):
        return self

    def end_of_epoch(self) -> bool:
        return False

    def state_dict(self):
        return None

    def load_state_dict(self, state):
        pass

    def close(self):
        pass


@register_task("pseudo")
class PseudoTask(Task):
    def load_dataset(self, split: str, **kwargs):
        self.datasets[split] = None
        return None

    def dataset(self, split: str):
        return None

    def get_batch_iterator(self, dataset, *, max_sentences=None, **kwargs):
        return PseudoIterator(max_sentences or self.cfg.batch_size or 1, self.cfg.tokens_per_sample, 10000)
