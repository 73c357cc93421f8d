"""Multiple-choice evaluation tasks scored by per-option log-likelihood (yoco/tasks/harness_eval.py:28-150,
harness_task.py:4-288, mmlu_task.py:4-92).

Each task reads ``<data_dir>/<dataname>`` (jsonl with ``ctx`` / ``label`` / ``choices`` / ``gold`` plus the raw
fields), turns every example into one (context, continuation) pair per option, and tokenises it as
``[BOS] + ctx + continuation`` with a loss mask over the continuation (the context is cut from the left when the pair
does not fit ``tokens_per_sample``). The option table below (dataname, class count, option builder) is the same
table as the reference's per-task classes, and the 57 MMLU subjects are registered as ``hendrycksTest-<subject>``.
"""
from __future__ import annotations

import json
import os
from typing import Callable, Dict, List, Tuple

import numpy as np
import torch

from ..registry import register_task
from .base import Task


def _fixed(answers: List[str]):
    def build(ex, n):
        return [ex["text"]] * n, list(answers), ex["label"]
    return build


def _choices_per_option(ex, n):
    return [ex["text"]] * len(ex["choices"]), [" " + c for c in ex["choices"]], ex["gold"]


def _choices_fixed_count(ex, n):
    return [ex["text"]] * n, [" " + c for c in ex["choices"]], ex["gold"]


def _copa(ex, n):
    return [ex["text"]] * n, [" " + ex["raw"]["choice1"], " " + ex["raw"]["choice2"]], ex["label"]


def _winogrande(ex, n):
    s = ex["raw"]["sentence"]
    cut = s.index("_")
    head = s[:cut].strip()
    ctx = [head + " " + ex["raw"]["option1"], head + " " + ex["raw"]["option2"]]
    return ctx, [" " + s[cut + 1:].strip()] * n, int(ex["raw"]["answer"]) - 1


def _truthful(key: str):
    def build(ex, n):
        choices = ex["raw"][key]["choices"]
        return [ex["text"]] * len(choices), [" " + c for c in choices], 0
    return build


def _record(ex, n):
    ents = ex["raw"]["entities"]
    return [ex["text"]] * len(ents), [f'  - {ex["raw"]["query"]}'.replace("@placeholder", e) for e in ents], 0


def _sciq(ex, n):
    r = ex["raw"]
    return ([ex["text"]] * n, [" " + r["distractor1"], " " + r["distractor2"], " " + r["distractor3"],
                               " " + r["correct_answer"]], 3)


# task name -> (file name, class_num, option builder)
HARNESS_TASKS: Dict[str, Tuple[str, int, Callable]] = {
    "harness_anli_r1": ("anli_r1", 3, _fixed([" True", " Neither", " False"])),
    "harness_anli_r2": ("anli_r2", 3, _fixed([" True", " Neither", " False"])),
    "harness_anli_r3": ("anli_r3", 3, _fixed([" True", " Neither", " False"])),
    "harness_boolq": ("boolq", 2, _fixed([" no", " yes"])),
    "harness_copa": ("copa", 2, _copa),
    "harness_openbookqa": ("openbookqa", 4, _choices_per_option),
    "harness_piqa": ("piqa", 2, _choices_per_option),
    "harness_rte": ("rte", 2, _fixed([" True", " False"])),
    "harness_wic": ("wic", 2, _fixed([" True", " False"])),
    "harness_winogrande": ("winogrande", 2, _winogrande),
    "harness_hellaswag": ("hellaswag", 4, _choices_fixed_count),
    "harness_arc_challenge": ("arc_challenge", 5, _choices_per_option),
    "harness_arc_easy": ("arc_easy", 5, _choices_per_option),
    "harness_record": ("record", 1, _record),
    "harness_truthfullqa_mc1": ("truthfulqa_mc", 1, _truthful("mc1_targets")),
    "harness_truthfullqa_mc2": ("truthfulqa_mc", 1, _truthful("mc2_targets")),
    "harness_arc_challenge_25s": ("arc_challenge_25s", 5, _choices_per_option),
    "harness_hellaswag_10s": ("hellaswag_10s", 4, _choices_fixed_count),
    "harness_sciq": ("sciq", 4, _sciq),
}

MMLU_SUBJECTS = [
    "abstract_algebra", "anatomy", "astronomy", "business_ethics", "clinical_knowledge", "college_biology",
    "college_chemistry", "college_computer_science", "college_mathematics", "college_medicine", "college_physics",
    "computer_security", "conceptual_physics", "econometrics", "electrical_engineering", "elementary_mathematics",
    "formal_logic", "global_facts", "high_school_biology", "high_school_chemistry", "high_school_computer_science",
    "high_school_european_history", "high_school_geography", "high_school_government_and_politics",
    "high_school_macroeconomics", "high_school_mathematics", "high_school_microeconomics", "high_school_physics",
    "high_school_psychology", "high_school_statistics", "high_school_us_history", "high_school_world_history",
    "human_aging", "human_sexuality", "international_law", "jurisprudence", "logical_fallacies", "machine_learning",
    "management", "marketing", "medical_genetics", "miscellaneous", "moral_disputes", "moral_scenarios", "nutrition",
    "philosophy", "prehistory", "professional_accounting", "professional_law", "professional_medicine",
    "professional_psychology", "public_relations", "security_studies", "sociology", "us_foreign_policy", "virology",
    "world_religions",
]
for _sub in MMLU_SUBJECTS:
    HARNESS_TASKS[f"hendrycksTest-{_sub}"] = (_sub, 4, _choices_fixed_count)


class HarnessDataset:
    """Tokenised options of one task: lists of src tokens, loss masks, label lengths (chars) and gold labels."""

    def __init__(self, name: str, tokenizer, data_dir: str, tokens_per_sample: int = 1024, verbose: bool = False):
        if name not in HARNESS_TASKS:
            raise KeyError(f"unknown harness task {name!r}")
        self.name = name
        self.dataname, self.class_num, self.build = HARNESS_TASKS[name]
        self.tokenizer, self.tokens_per_sample = tokenizer, tokens_per_sample
        self.examples = self._load(os.path.join(data_dir, self.dataname))
        self.verbose = verbose

    @staticmethod
    def _load(path: str):
        out = []
        with open(path, encoding="utf-8") as f:
            for line in f:
                if not line.strip():
                    continue
                obj = json.loads(line)
                out.append({"text": obj.get("ctx"), "label": obj.get("label"), "choices": obj.get("choices", []),
                            "gold": obj.get("gold"), "raw": obj})
        return out

    def get_data_for_evaluation(self):
        src, masks, label_len, labels = [], [], [], []
        cut = 0
        tps = self.tokens_per_sample
        for ex in self.examples:
            ctxs, conts, label = self.build(ex, self.class_num)
            for ctx, cont in zip(ctxs, conts):
                ctx_ids = self.tokenizer.encode(ctx)
                cont_ids = self.tokenizer.encode(ctx + cont)[len(ctx_ids):]
                if len(ctx_ids) + len(cont_ids) + 1 >= tps:
                    cut += 1
                    ctx_ids = ctx_ids[-(tps - len(cont_ids) - 1):]
                src.append([self.tokenizer.bos_id] + ctx_ids + cont_ids)
                masks.append([False] * (len(ctx_ids) + 1) + [True] * len(cont_ids))
                label_len.append(len(cont.strip()))
                labels.append(label)
        if cut and self.verbose:
            print(f"cut {cut} examples")
        return src, masks, np.array(label_len), np.array(labels)


def collate_options(src, masks, label_len, labels, pad_id: int):
    """Right-pad a list of option sequences into one batch dict."""
    n = len(src)
    width = max(len(s) for s in src)
    tok = torch.full((n, width), pad_id, dtype=torch.long)
    m = torch.zeros((n, width), dtype=torch.bool)
    for i, (s, k) in enumerate(zip(src, masks)):
        tok[i, :len(s)] = torch.tensor(s, dtype=torch.long)
        m[i, :len(k)] = torch.tensor(k, dtype=torch.bool)
    return {"net_input": {"src_tokens": tok, "gpt_loss_mask": m,
                          "label_length": torch.as_tensor(label_len, dtype=torch.long),
                          "src_lengths": torch.tensor([len(s) for s in src])},
            "targets": torch.as_tensor(labels, dtype=torch.long), "nsentences": n,
            "ntokens": int(sum(len(s) for s in src))}


@register_task("harness_eval")
class HarnessEval(Task):
    def __init__(self, cfg, tokenizer):
        super().__init__(cfg, tokenizer)
        self.harness_task = HarnessDataset(cfg.eval_data, tokenizer, cfg.data_dir, cfg.tokens_per_sample)

    def load_dataset(self, split: str, **kwargs):
        self.datasets[split] = self.harness_task.get_data_for_evaluation()
        return self.datasets[split]

    def get_batch_iterator(self, dataset, *, max_sentences=None, num_shards: int = 1, shard_id: int = 0, **kwargs):
        """Sequential batches of whole examples (a multiple of the class count per batch); shards take every
        num_shards-th batch."""
        src, masks, label_len, labels = dataset
        per = max(1, (max_sentences or self.harness_task.class_num) // self.harness_task.class_num)
        step = per * self.harness_task.class_num
        batches = []
        for i in range(0, len(src), step):
            batches.append(collate_options(src[i:i + step], masks[i:i + step], label_len[i:i + step],
                                           labels[i:i + step], self.tokenizer.pad_id))
        return iter(batches[shard_id::num_shards])
