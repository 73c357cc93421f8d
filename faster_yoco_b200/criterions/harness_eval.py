"""Multiple-choice scoring (yoco/criterions/harness_eval.py:9-86): summed NLL of each option's continuation tokens;
the prediction is the argmin over the options of an example (``accuracy``) or of the NLL divided by the
continuation's character length (``accuracy_norm``)."""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ..registry import register_criterion


@register_criterion("harness_eval")
class HarnessEvalCriterion:
    def __init__(self, task):
        self.task = task
        self.padding_idx = task.target_dictionary.pad()

    @torch.no_grad()
    def __call__(self, model, sample, reduce: bool = True):
        model.eval()
        ni = sample["net_input"]
        logits, _ = model(ni["src_tokens"])
        logits = logits[:, :-1, :]
        targets = ni["src_tokens"][:, 1:]
        mask = ni["gpt_loss_mask"][:, 1:]
        nll = F.cross_entropy(logits.float().reshape(-1, logits.size(-1)), targets.reshape(-1), reduction="none",
                              ignore_index=self.padding_idx).view(targets.size(0), -1)
        nll = nll * mask.to(nll.dtype)
        per_option = nll.sum(-1)
        per_option_norm = per_option / ni["label_length"].to(per_option.device).float()
        k = self.task.harness_task.class_num
        if per_option.numel() % k:
            raise ValueError(f"batch of {per_option.numel()} options is not a multiple of {k}")
        gold = sample["targets"].view(-1, k)[:, 0].to(per_option.device)
        pred = per_option.view(-1, k).argmin(1)
        pred_norm = per_option_norm.view(-1, k).argmin(1)
        log = {"loss": 0, "nsentences": pred.numel(), "sample_size": pred.numel(),
               "ncorrect": int((pred == gold).sum()), "ncorrect_norm": int((pred_norm == gold).sum())}
        return per_option, sample["ntokens"], log

    @staticmethod
    def reduce_metrics(logs):
        n = sum(l.get("nsentences", 0) for l in logs) or 1
        return {"loss": round(sum(l.get("loss", 0) for l in logs) / n, 3),
                "accuracy": round(100.0 * sum(l.get("ncorrect", 0) for l in logs) / n, 2),
                "accuracy_norm": round(100.0 * sum(l.get("ncorrect_norm", 0) for l in logs) / n, 2)}
