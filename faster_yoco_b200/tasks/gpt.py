"""GPT pretraining task: packed jsonl shards through :class:`~faster_yoco_b200.data.lm_loader.LMLoader`
(yoco/tasks/gpt.py:16-176). ``load_dataset(split)`` reads ``<data>/json/<split>.json`` (the list of sources)."""
from __future__ import annotations

import json
import os
from types import SimpleNamespace

from ..data.lm_loader import LMLoader
from ..registry import register_task
from .base import Task, TaskConfig


@register_task("gpt")
class GPTPretrainingTask(Task):
    def load_dataset(self, split: str, epoch: int = 1, combine: bool = False, **kwargs):
        if self.cfg.data is None:
            raise FileNotFoundError("no data directory given")
        with open(os.path.join(self.cfg.data, "json", f"{split}.json")) as f:
            data = json.load(f)
        self.datasets[split] = SimpleNamespace(data=data, data_dir=self.cfg.data, shuffle=split == "train")
        return self.datasets[split]

    def get_batch_iterator(self, dataset, *, max_sentences=None, seed: int = 1, num_shards: int = 1,
                           shard_id: int = 0, epoch: int = 1, prefetch: int = 10, **kwargs):
        return LMLoader(dataset.data, dataset.data_dir, self.tokenizer,
                        tokens_per_sample=self.cfg.tokens_per_sample,
                        batch_size=max_sentences or self.cfg.batch_size or 1, seed=seed, num_shards=num_shards,
                        shard_id=shard_id,
                        batch_read_ahead=self.cfg.batch_read_ahead if dataset.shuffle else 0,
                        pad_to_max_len=self.cfg.pad_to_max_len, prefetch=prefetch,
                        absolute_path=self.cfg.absolute_path, endless=dataset.shuffle)
