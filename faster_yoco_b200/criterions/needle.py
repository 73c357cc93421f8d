"""Passkey retrieval over long contexts (yoco/criterions/needle_haystack.py:47-169, multi_needle.py:53-181).

For every context length ``interval, 2 interval, ..., tokens_per_sample`` (150 tokens kept for the question) and
every depth, a haystack of essay lines (files under ``needle_file_path``) gets one needle sentence -- or several
for ``multi_needle``, whose question asks about the last needle before the depth point -- and the model answers by
greedy generation (chunked prefill). Accuracy = fraction of trials whose output contains the number. The prompt
templates, the city list and the seeds (0 for one needle, 42 for several) are the reference's, so the same
haystacks come out for the same essays and tokenizer.
"""
from __future__ import annotations

import os
import random
from typing import Dict, List, Optional

import torch

from ..eval.generate import generate
from ..registry import register_criterion

PROMPT = ("There is a special magic number inside a lot of irrelevant text. Find it and memorize them. "
          "I will quiz you about the magic number there. {context} ")
QUESTION = "What is the special magic {city} number? The special magic {city} number is "
NEEDLE_ONE = "The special magic {city} number is {rnd_number} . "
NEEDLE_MULTI = "The special magic {city} number is: {rnd_number}"
CITIES = [
    'Chicago', 'Yangon', 'Antananarivo', 'Colombo', 'Almaty', 'Sydney', 'Chicago', 'Mexico City',
    'Seattle', 'Lagos', 'Amsterdam', 'Belgrade', 'Cairo', 'Baghdad', 'Damascus', 'Kigali', 'Dakar',
    'Dakar', 'Sofia', 'Kigali', 'Victoria', 'Tashkent', 'Mumbai', 'Barcelona', 'Almaty', 'Amman',
    'Toronto', 'Bratislava', 'Johannesburg', 'Thimphu', 'Bangkok', 'Santiago', 'Cairo', 'San Francisco',
    'Lagos', 'Amsterdam', 'Paris', 'Rabat', 'Santiago', 'Copenhagen', 'Madrid', 'Kigali',
    'Ho Chi Minh City', 'Sarajevo', 'Delhi', 'Istanbul', 'Ho Chi Minh City', 'Khartoum', 'Helsinki',
    'Doha', 'Istanbul', 'Kuala Lumpur', 'Budapest', 'Shanghai', 'Moscow', 'Los Angeles', 'Oslo',
    'Johannesburg', 'Berlin', 'Bangalore', 'Tokyo', 'Melbourne', 'Barcelona', 'Chicago', 'Port Louis',
    'Lisbon', 'Nairobi', 'Kampala', 'Lima', 'Maputo', 'Vancouver', 'Dubai', 'Khartoum', 'Jakarta',
    'Madrid', 'Yerevan', 'Beirut', 'Athens', 'Chicago', 'Paris', 'Bucharest', 'Copenhagen', 'Brussels',
    'Damascus', 'Seattle', 'Los Angeles', 'Yerevan', 'Victoria', 'Tunis', 'Astana', 'Seoul',
    'Buenos Aires', 'Bangkok', 'Colombo', 'Brussels', 'Khartoum', 'Doha', 'San Francisco', 'Vienna', 'Jakarta',
]


def random_partition(total: int, n: int) -> List[int]:
    """n positive parts summing to total (sorted random cut points)."""
    cuts = sorted(random.sample(range(1, total), n - 1))
    edges = [0] + cuts + [total]
    return [edges[i + 1] - edges[i] for i in range(n)]


class _Haystack:
    def __init__(self, needle_file_path: str, tokenizer):
        self.dir = needle_file_path
        self.essays = sorted(os.listdir(needle_file_path)) * 5000 if os.path.isdir(needle_file_path) else []
        self.tok = tokenizer
        self._cache: Dict[str, List[str]] = {}

    def garbage(self, length: int) -> str:
        """Whole essay lines (each followed by a space) until the next one would exceed `length` tokens."""
        text, n = [], 0
        if not self.essays:
            raise FileNotFoundError(f"no essays under {self.dir}")
        while True:
            name = random.choice(self.essays)
            if name not in self._cache:
                with open(os.path.join(self.dir, name)) as f:
                    self._cache[name] = f.read().splitlines()
            for line in self._cache[name]:
                k = len(self.tok.encode(line + " "))
                if n + k > length:
                    return "".join(text)
                text.append(line + " ")
                n += k


class _NeedleBase:
    seed = 0
    trials = 10

    def __init__(self, task, tokens_per_sample: int = 16384, interval: int = 1024,
                 needle_file_path: str = "", generate_tokens: int = 20, chunk_length: int = 32768,
                 yoco: bool = True, verbose: bool = False):
        self.task = task
        self.tokens_per_sample, self.interval = tokens_per_sample, interval
        self.hay = _Haystack(needle_file_path, task.tokenizer)
        self.generate_tokens, self.chunk_length, self.yoco, self.verbose = generate_tokens, chunk_length, yoco, verbose

    def depths(self, all_length: int):
        raise NotImplementedError

    def prompt(self, prefix: int, suffix: int):
        raise NotImplementedError

    @torch.no_grad()
    def __call__(self, model, sample=None, reduce: bool = True, device=None):
        model.eval()
        dev = device or next(model.parameters()).device
        tok = self.task.tokenizer
        random.seed(self.seed)
        results = {}
        for ctx_len in range(self.interval, self.tokens_per_sample + 1, self.interval):
            all_length = ctx_len - 150
            row = []
            for prefix, suffix in self.depths(all_length):
                hits = 0
                for _ in range(self.trials):
                    text, answer = self.prompt(prefix, suffix)
                    ids = torch.tensor([tok.encode(text, bos=True)], device=dev)
                    out = generate(model, ids, tok, self.generate_tokens, self.chunk_length, yoco=self.yoco)
                    pred = tok.decode(out[0, ids.shape[1]:].tolist())
                    if self.verbose:
                        print("Answer:", answer, "Pred:", pred)
                    hits += answer in pred
                row.append(hits / self.trials)
            results[ctx_len] = row
        return 0, 1, {"loss": 0, "retrieval": results}

    @staticmethod
    def reduce_metrics(logs):
        return {"retrieval": [l.get("retrieval") for l in logs]}


@register_criterion("needle_haystack")
class NeedleHaystackCriterion(_NeedleBase):
    seed, trials = 0, 10

    def depths(self, all_length):
        for d in range(0, 11):
            p = int(all_length * d / 10)
            yield p, all_length - p

    def prompt(self, prefix, suffix):
        city = random.choice(CITIES)
        number = random.randint(1, 50000)
        pre = self.hay.garbage(prefix)
        post = self.hay.garbage(suffix)
        ctx = "\n".join([pre, NEEDLE_ONE.format(city=city, rnd_number=number), post, QUESTION.format(city=city)])
        return PROMPT.format(context=ctx), str(number)


@register_criterion("multi_needle")
class MultiNeedleCriterion(_NeedleBase):
    seed, trials = 42, 5

    def __init__(self, task, needle_num: int = 4, **kw):
        super().__init__(task, **kw)
        self.needle_num = needle_num

    def depths(self, all_length):
        for d in range(1, 11):
            p = int(all_length * d / 11)
            yield p, all_length - p

    def prompt(self, prefix, suffix):
        n = self.needle_num
        if n > 1:
            first = random.randint(1, n - 1)
            first_parts = random_partition(prefix, first)
            second_parts = random_partition(suffix, n + 1 - first)
            final = second_parts.pop()
        else:
            first_parts, second_parts, final = [prefix], [], suffix
        cities = random.sample(CITIES, n)
        lines = []
        for length in first_parts:
            lines.append(self.hay.garbage(length))
            city = cities.pop()
            number = random.randint(1, 50000)
            lines.append(NEEDLE_MULTI.format(city=city, rnd_number=number))
        question, answer = QUESTION.format(city=city), number
        for length in second_parts:
            lines.append(self.hay.garbage(length))
            city = cities.pop()
            number = random.randint(1, 50000)
            lines.append(NEEDLE_MULTI.format(city=city, rnd_number=number))
        lines.append(self.hay.garbage(final))
        lines.append(question)
        return PROMPT.format(context="\n".join(lines)), str(answer)
