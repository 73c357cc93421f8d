"""Device-resident meters: nothing here makes the host wait for the GPU until a log line is due.

Mirrors the fairseq meters the reference logs (loss in bits = loss_sum / sample_size / ln 2, ppl, wpb, wps, bsz, ups,
gnorm, clip, train_wall; yoco/tasks/trainer_nosync.py:145-216) with the per-update values kept as GPU tensors and
summed on the GPU; ``flush()`` reads them back once per log interval.
"""
from __future__ import annotations

import math
import time
from typing import Dict, Optional

import torch


class DeviceMeters:
    def __init__(self, device):
        self.device = device
        self.keys = ["loss_sum", "sample_size", "ntokens", "nsentences", "gnorm", "clip", "updates"]
        self.acc = torch.zeros(len(self.keys), dtype=torch.float64, device=device)
        self.t0 = time.perf_counter()
        self.total_updates = 0

    def update(self, loss_sum, sample_size, ntokens, nsentences, gnorm, clip_norm: float):
        vals = torch.stack([
            loss_sum.double().reshape(()), sample_size.double().reshape(()),
            torch.as_tensor(float(ntokens), dtype=torch.float64, device=self.device),
            torch.as_tensor(float(nsentences), dtype=torch.float64, device=self.device),
            gnorm.double().reshape(()),
            (gnorm > clip_norm).double().reshape(()) * 100.0 if clip_norm > 0 else gnorm.new_zeros(()).double(),
            torch.ones((), dtype=torch.float64, device=self.device),
        ])
        self.acc += vals
        self.total_updates += 1

    def flush(self) -> Dict[str, float]:
        v = self.acc.cpu().tolist()
        self.acc.zero_()
        d = dict(zip(self.keys, v))
        dt = time.perf_counter() - self.t0
        self.t0 = time.perf_counter()
        n = max(d["updates"], 1.0)
        loss = d["loss_sum"] / max(d["sample_size"], 1.0) / math.log(2)
        return {
            "loss": round(loss, 3), "ppl": round(2 ** loss, 2) if loss < 100 else float("inf"),
            "wpb": round(d["ntokens"] / n, 1), "bsz": round(d["nsentences"] / n, 1),
            "wps": round(d["ntokens"] / dt, 1) if dt > 0 else 0.0, "ups": round(n / dt, 2) if dt > 0 else 0.0,
            "gnorm": round(d["gnorm"] / n, 3), "clip": round(d["clip"] / n, 1), "num_updates": self.total_updates,
        }


def format_log(stats: Dict[str, float], epoch: int = 1, fmt: str = "simple") -> str:
    """One training log line in fairseq's ``--log-format``: ``simple`` (``epoch 001: loss 3.1 | ...``, also used
    for ``tqdm``), ``json`` (one JSON object per line) or ``none`` (empty: nothing to print)."""
    if fmt == "none":
        return ""
    if fmt == "json":
        import json
        return json.dumps(dict({"epoch": epoch}, **{k: (round(v, 4) if isinstance(v, float) else v)
                                                   for k, v in stats.items()}))
    body = " | ".join(f"{k} {v}" for k, v in stats.items())
    return f"epoch {epoch:03d}: {body}"
