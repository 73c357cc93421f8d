"""Packed language-model loader (yoco/tasks/data/lm_loader.py, basic_loader.py).

Pipeline per data source (``{"name", "weight" | "count", "source": [files]}``; ``source`` defaults to the file list
in ``<data_dir>/json/<name>.json``):

1. the file list repeated 50 times and shuffled with ``Random(str(seed))``, cut into contiguous chunks, one per rank;
2. each jsonl file read and tokenised document by document: a document splits on blank lines, then on lines; each
   line is encoded with its trailing newline(s), and the document's last piece gets EOS (``_doc_to_ids``);
3. the pieces of a file packed into BOS-started samples of ``tokens_per_sample + 1`` ids: the piece that overflows
   a sample fills it up to its end (the rest of that piece is dropped) and the next sample starts with BOS alone; the
   partly filled sample at the end of a file is dropped;
4. sources multiplexed by weight with ``Random(seed + n)`` for the n-th sample;
5. blockwise shuffle (``batch_read_ahead`` samples per block, each block shuffled with ``Random(str(seed))``), fixed
   batches of ``batch_size``, collate: ``src_tokens = ids[:-1]``, ``target = ids[1:]`` (pad 1 up to
   ``tokens_per_sample`` when ``pad_to_max_len``), ``ntokens = sum(len(ids))`` (2049 for a full sample);
6. a prefetch thread; the loader never ends (a source restarts when exhausted).

``state_dict()`` / ``load_state_dict()`` resume at exactly the next batch.
"""
from __future__ import annotations

import json
import os
from random import Random
from typing import Dict, List, Optional

import numpy as np
import torch

from . import iterators as it


def doc_to_ids(text: str, tokenizer) -> List[List[int]]:
    pieces: List[List[int]] = []
    lines = text.split("\n\n")
    for li, line in enumerate(lines):
        suffix = "\n\n" if li != len(lines) - 1 else ""
        if not line:
            continue
        sub = line.split("\n")
        for si, s in enumerate(sub):
            if not s or len(s) > 200000:
                continue
            pieces.append(tokenizer.encode(s + suffix) if si == len(sub) - 1 else tokenizer.encode(s + "\n"))
    if pieces:
        pieces[-1].append(tokenizer.eos_id)
    return pieces


def pack(pieces: List[List[int]], bos: int, tokens_per_sample: int) -> List[List[int]]:
    out, doc = [], [bos]
    for ids in pieces:
        if len(doc) + len(ids) > tokens_per_sample + 1:
            doc.extend(ids)
            out.append(doc[:tokens_per_sample + 1])
            doc = [bos]
        else:
            doc.extend(ids)
    return out


def read_jsonl_samples(path: str, tokenizer, tokens_per_sample: int) -> List[List[int]]:
    if not os.path.exists(path):
        return []
    pieces: List[List[int]] = []
    with open(path, encoding="utf8") as f:
        for line in f.read().strip().split("\n"):
            if not line:
                continue
            try:
                obj = json.loads(line)
            except json.JSONDecodeError:
                continue
            text = obj.get("text") or obj.get("content") or "\n".join(obj.get("raw_content_lines", []))
            if text:
                pieces.extend(doc_to_ids(text, tokenizer))
    return pack(pieces, tokenizer.bos_id, tokens_per_sample)


class LMLoader:
    def __init__(self, data: List[Dict], data_dir: str, tokenizer, *, tokens_per_sample: int, batch_size: int,
                 seed: int = 1, num_shards: int = 1, shard_id: int = 0, batch_read_ahead: int = 1000,
                 pad_to_max_len: bool = True, epochs: int = 50, prefetch: int = 10, absolute_path: bool = False,
                 endless: bool = True):
        """endless=False (evaluation): one pass over the files in their listed order (no repetition, no shuffle),
        then StopIteration."""
        self.endless = endless
        self.data, self.data_dir, self.tok = data, data_dir, tokenizer
        self.tps, self.bsz, self.seed = tokens_per_sample, batch_size, str(seed)
        self.num_shards, self.shard_id = num_shards, shard_id
        self.read_ahead, self.pad_to_max_len, self.epochs = batch_read_ahead, pad_to_max_len, epochs
        self.absolute_path = absolute_path
        self._iter = it.PrefetchIterator(self._batches(), prefetch) if prefetch > 0 else self._batches()

    # ------------------------------------------------------------------------------------------------------------
    def _source_files(self, d: Dict) -> List[str]:
        if d.get("source"):
            return list(d["source"])
        path = os.path.join(self.data_dir, "json", f"{d['name']}.json")
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        with open(path, encoding="utf8") as f:
            return json.load(f)

    def _lines(self, d: Dict):
        files = self._source_files(d)
        if not self.endless:
            return it.SelectManyIterator(it.chunked_source(list(files), self.num_shards, self.shard_id), self._read)

        def make(epoch: int):
            items = files * self.epochs
            Random(self.seed).shuffle(items)
            chunk = it.chunked_source(items, self.num_shards, self.shard_id)
            return it.SelectManyIterator(chunk, self._read)
        return it.RepeatIterator(make)

    def _read(self, f: str) -> List[List[int]]:
        path = f if self.absolute_path else os.path.join(self.data_dir, f)
        return read_jsonl_samples(path, self.tok, self.tps)

    def _batches(self):
        sources = [self._lines(d) for d in self.data]
        if len(sources) == 1:
            lines = sources[0]
        elif not self.endless:
            lines = it.ChainIterator(sources)          # evaluation: every source once, in order
        else:
            weights = [float(d["weight"]) if "weight" in d else int(d["count"]) for d in self.data]
            lines = it.MultiplexIterator(it.WeightNoRandomStateIterator(weights, int(self.seed)), sources)
        if self.read_ahead > 0:
            lines = it.fixed_blockwise_shuffle(lines, self.read_ahead, self.seed)
        return it.MapIterator(it.FixedBatchIterator(lines, self.bsz), self._collate)

    def _collate(self, batch: List[List[int]]) -> Dict:
        width = (self.tps + 1 if self.pad_to_max_len else max(len(x) for x in batch)) - 1
        src = np.full((len(batch), width), self.tok.pad_id, dtype=np.int64)
        tgt = np.full((len(batch), width), self.tok.pad_id, dtype=np.int64)
        for i, ids in enumerate(batch):
            src[i, :len(ids) - 1] = ids[:-1]
            tgt[i, :len(ids) - 1] = ids[1:]
        return {"src_tokens": torch.from_numpy(src), "target": torch.from_numpy(tgt),
                "nsentences": len(batch), "ntokens": sum(len(x) for x in batch)}

    # ------------------------------------------------------------------------------------------------------------
    def __iter__(self):
        return self

    def __next__(self):
        return next(self._iter)

    def __len__(self):
        return 819200000

    def state_dict(self):
        return self._iter.getstate()

    def load_state_dict(self, state):
        self._iter.setstate(state)

    def close(self):
        self._iter.close()
