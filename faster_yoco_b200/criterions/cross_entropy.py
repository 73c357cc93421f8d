"""Language-model cross-entropy (fairseq's ``CrossEntropyCriterion`` as the reference trains with it, with the
fused CE of yoco/tasks/fused_ce.py:62-116): fp32 sum of ``lse - logit[target]`` over non-pad targets; the sample size
is ``ntokens``; the logged loss is in bits (``loss_sum / sample_size / ln 2``)."""
from __future__ import annotations

import math

import torch

from .. import ops
from ..registry import register_criterion


@register_criterion("cross_entropy")
class CrossEntropyCriterion:
    def __init__(self, task=None, padding_idx: int = 1, sentence_avg: bool = False):
        self.task = task
        self.padding_idx = task.target_dictionary.pad() if task is not None else padding_idx
        self.sentence_avg = sentence_avg

    def __call__(self, model, sample, reduce: bool = True):
        src = sample["net_input"]["src_tokens"] if "net_input" in sample else sample["src_tokens"]
        logits, _ = model(src)
        V = logits.shape[-1]
        loss = ops.cross_entropy(logits.reshape(-1, V), sample["target"].reshape(-1), self.padding_idx)
        sample_size = sample.get("nsentences", src.size(0)) if self.sentence_avg else sample["ntokens"]
        log = {"loss": loss.detach(), "ntokens": sample["ntokens"], "nsentences": sample.get("nsentences", src.size(0)),
               "sample_size": sample_size}
        return loss, sample_size, log

    @staticmethod
    def reduce_metrics(logs):
        loss = sum(float(l.get("loss", 0)) for l in logs)
        ss = sum(l.get("sample_size", 0) for l in logs) or 1
        bits = loss / ss / math.log(2)
        return {"loss": round(bits, 3), "ppl": round(2 ** bits, 2),
                "ntokens": sum(l.get("ntokens", 0) for l in logs)}
