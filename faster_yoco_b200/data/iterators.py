"""Checkpointable iterator pipeline (the infinibatch stages the reference's loader is built from:
yoco/tasks/data/lm_loader.py, basic_loader.py, utils.py).

Every stage exposes ``getstate()`` / ``setstate(state)``; the state of a pipeline is the nested state of its last
stage, so a resumed loader continues with exactly the next batch.
"""
from __future__ import annotations

import copy
import math
import queue
import threading
from random import Random
from typing import Any, Callable, Iterable, List, Optional


class CheckpointableIterator:
    def __iter__(self):
        return self

    def __next__(self):
        raise NotImplementedError

    def getstate(self):
        raise NotImplementedError

    def setstate(self, state):
        raise NotImplementedError

    def close(self):
        pass


class NativeCheckpointableIterator(CheckpointableIterator):
    """Over an in-memory list; state = position."""

    def __init__(self, items: List[Any]):
        self.items = items
        self.pos = 0

    def __next__(self):
        if self.pos >= len(self.items):
            raise StopIteration
        item = self.items[self.pos]
        self.pos += 1
        return item

    def getstate(self):
        return {"pos": self.pos}

    def setstate(self, state):
        self.pos = state["pos"] if state else 0


def chunked_source(items: List[Any], num_instances: int = 1, instance_rank: int = 0) -> NativeCheckpointableIterator:
    """Contiguous chunk `instance_rank` of ceil(len / num_instances) items (sharding by rank)."""
    size = math.ceil(len(items) / num_instances)
    return NativeCheckpointableIterator(items[instance_rank * size:(instance_rank + 1) * size])


class MapIterator(CheckpointableIterator):
    def __init__(self, source: CheckpointableIterator, fn: Callable):
        self.source, self.fn = source, fn

    def __next__(self):
        return self.fn(next(self.source))

    def getstate(self):
        return self.source.getstate()

    def setstate(self, state):
        self.source.setstate(state)


class SelectManyIterator(CheckpointableIterator):
    """Flattens fn(item) for each source item; state = (source state before the current collection, index)."""

    def __init__(self, source: CheckpointableIterator, fn: Callable[[Any], Iterable]):
        self.source, self.fn = source, fn
        self.setstate(None)

    def __next__(self):
        while self._cur is None or self._i >= len(self._cur):
            self._src_state = self.source.getstate()
            self._cur = list(self.fn(next(self.source)))
            self._i = 0
        item = self._cur[self._i]
        self._i += 1
        return item

    def getstate(self):
        return {"src": copy.deepcopy(self._src_state), "i": self._i}

    def setstate(self, state):
        self._cur, self._i = None, 0
        if state is None:
            self.source.setstate(None)
            self._src_state = self.source.getstate()
            return
        self.source.setstate(state["src"])
        self._src_state = copy.deepcopy(state["src"])
        if state["i"] > 0:
            self._cur = list(self.fn(next(self.source)))
            self._i = state["i"]


class FixedBatchIterator(CheckpointableIterator):
    def __init__(self, source: CheckpointableIterator, batch_size: int):
        self.source, self.batch_size = source, batch_size

    def __next__(self):
        batch = []
        for _ in range(self.batch_size):
            try:
                batch.append(next(self.source))
            except StopIteration:
                break
        if not batch:
            raise StopIteration
        return batch

    def getstate(self):
        return self.source.getstate()

    def setstate(self, state):
        self.source.setstate(state)


def fixed_blockwise_shuffle(source: CheckpointableIterator, block_size: int, seed) -> CheckpointableIterator:
    """Group `block_size` consecutive items, shuffle each block with a fresh Random(seed), flatten
    (yoco/tasks/data/utils.py:97-121)."""
    def shuffle_block(block):
        Random(seed).shuffle(block)
        return block
    return SelectManyIterator(MapIterator(FixedBatchIterator(source, block_size), shuffle_block), lambda b: b)


class WeightNoRandomStateIterator(CheckpointableIterator):
    """Source index for the n-th item: Random(seed + n).choices(range(k), weights) (no carried RNG state)."""

    def __init__(self, weights: List[float], seed):
        self.weights, self.seed = list(weights), int(seed)
        self.n = 0

    def __next__(self):
        idx = Random(self.seed + self.n).choices(range(len(self.weights)), self.weights)[0]
        self.n += 1
        return idx

    def getstate(self):
        return {"n": self.n}

    def setstate(self, state):
        self.n = state["n"] if state else 0


class WeightIterator(CheckpointableIterator):
    """Source index drawn from ONE Random(seed) stream whose state is checkpointed (the carried-state variant of
    WeightNoRandomStateIterator; yoco/tasks/data/utils.py:65-95)."""

    def __init__(self, weights: List[float], seed):
        self.weights, self.seed = list(weights), seed
        self.setstate(None)

    def __next__(self):
        if self._rng is None:
            self._rng = Random(self.seed)
            if self._rng_state is not None:
                self._rng.setstate(self._rng_state)
        idx = self._rng.choices(range(len(self.weights)), self.weights)[0]
        self._rng_state = self._rng.getstate()
        return idx

    def getstate(self):
        return {"random_state": self._rng_state}

    def setstate(self, state):
        self._rng_state = state["random_state"] if state else None
        self._rng = None


class IndexIterator(CheckpointableIterator):
    """0, 1, ..., num - 1, 0, 1, ... with the count of yielded items as its state (utils.py:124-144)."""

    def __init__(self, num: int):
        self.num = num
        self.setstate(None)

    def __next__(self):
        item = self.n % self.num
        self.n += 1
        return item

    def getstate(self):
        return {"n": self.n}

    def setstate(self, state):
        self.n = state["n"] if state else 0


class MultiplexIterator(CheckpointableIterator):
    def __init__(self, control: CheckpointableIterator, sources: List[CheckpointableIterator]):
        self.control, self.sources = control, sources

    def __next__(self):
        return next(self.sources[next(self.control)])

    def getstate(self):
        return {"control": self.control.getstate(), "sources": [s.getstate() for s in self.sources]}

    def setstate(self, state):
        self.control.setstate(state["control"] if state else None)
        for i, s in enumerate(self.sources):
            s.setstate(state["sources"][i] if state else None)


class ChainIterator(CheckpointableIterator):
    """The items of each source in turn (evaluation passes over several sources)."""

    def __init__(self, sources: List[CheckpointableIterator]):
        self.sources = sources
        self.setstate(None)

    def __next__(self):
        while self.i < len(self.sources):
            try:
                return next(self.sources[self.i])
            except StopIteration:
                self.i += 1
        raise StopIteration

    def getstate(self):
        return {"i": self.i, "src": self.sources[self.i].getstate() if self.i < len(self.sources) else None}

    def setstate(self, state):
        self.i = state["i"] if state else 0
        for j, src in enumerate(self.sources):
            src.setstate(state["src"] if (state and j == self.i) else None)


class RepeatIterator(CheckpointableIterator):
    """Restart the source when it is exhausted (the loader 'never ends'); state counts passes."""

    def __init__(self, make_source: Callable[[int], CheckpointableIterator]):
        self.make_source = make_source
        self.setstate(None)

    def __next__(self):
        while True:
            try:
                return next(self.source)
            except StopIteration:
                self.epoch += 1
                self.source = self.make_source(self.epoch)

    def getstate(self):
        return {"epoch": self.epoch, "src": self.source.getstate()}

    def setstate(self, state):
        self.epoch = state["epoch"] if state else 0
        self.source = self.make_source(self.epoch)
        self.source.setstate(state["src"] if state else None)


class PrefetchIterator(CheckpointableIterator):
    """Background thread filling a bounded buffer; each buffered item carries the source state after it, so the
    checkpoint is exactly the position of the last item handed out."""

    def __init__(self, source: CheckpointableIterator, buffer_size: int = 10):
        self.source, self.buffer_size = source, buffer_size
        self._thread = None
        self.setstate(None)

    def _start(self):
        self._q: "queue.Queue" = queue.Queue(self.buffer_size)
        self._stop = threading.Event()

        def run():
            try:
                while not self._stop.is_set():
                    item = next(self.source)
                    self._q.put((item, copy.deepcopy(self.source.getstate())))
            except StopIteration:
                self._q.put(None)
            except Exception as e:  # surfaced on the consumer side
                self._q.put(e)
        self._thread = threading.Thread(target=run, daemon=True)
        self._thread.start()

    def __next__(self):
        got = self._q.get()
        if got is None:
            raise StopIteration
        if isinstance(got, Exception):
            raise got
        item, self._state = got
        return item

    def getstate(self):
        return self._state

    def setstate(self, state):
        self.close()
        self.source.setstate(state)
        self._state = copy.deepcopy(self.source.getstate())
        self._start()

    def close(self):
        if self._thread is not None:
            self._stop.set()
            for _ in range(1000):                  # keep draining until the producer notices the stop flag
                try:
                    while True:
                        self._q.get_nowait()
                except queue.Empty:
                    pass
                self._thread.join(timeout=0.01)
                if not self._thread.is_alive():
                    break
            self._thread = None
