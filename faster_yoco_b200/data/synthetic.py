"""Synthetic batches: uniform-random token ids of the benchmark shape (no dataset or tokenizer file is reachable
offline). Batches follow the reference collate layout (yoco/tasks/data/lm_loader.py:131-159): ``src_tokens`` and
``target`` [B, L] int64 (target = source shifted by one), ``ntokens`` = B * (L + 1), ``nsentences`` = B."""
from __future__ import annotations

import torch


class SyntheticLM:
    def __init__(self, vocab: int, seq_len: int, batch: int, seed: int = 1, rank: int = 0, pin: bool = False):
        self.vocab, self.seq_len, self.batch = vocab, seq_len, batch
        self.gen = torch.Generator().manual_seed(seed * 1000003 + rank)
        self.pin = pin

    def __iter__(self):
        return self

    def __next__(self):
        ids = torch.randint(0, self.vocab, (self.batch, self.seq_len + 1), generator=self.gen, dtype=torch.int64)
        src, tgt = ids[:, :-1].contiguous(), ids[:, 1:].contiguous()
        if self.pin:
            src, tgt = src.pin_memory(), tgt.pin_memory()
        return {"src_tokens": src, "target": tgt, "ntokens": self.batch * (self.seq_len + 1),
                "nsentences": self.batch}

    def state_dict(self):
        return {"gen": self.gen.get_state()}

    def load_state_dict(self, sd):
        self.gen.set_state(sd["gen"])
