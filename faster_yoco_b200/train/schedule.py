"""Learning-rate schedule: fairseq ``polynomial_decay`` (the reference recipe's ``--lr-scheduler``).

fairseq sets the warm-up factor ``1 / warmup_updates`` at construction and calls ``step_update(num_updates)`` after
every update, so the update that follows ``n`` completed updates runs with ``lr(max(n, 1))`` during warm-up:
updates 1 and 2 both use lr/warmup.
"""
from __future__ import annotations

from ..ops.reference import polynomial_decay_lr


class PolynomialDecaySchedule:
    def __init__(self, lr: float, warmup_updates: int, total_num_update: int, end_learning_rate: float = 0.0,
                 power: float = 1.0):
        self.base_lr, self.warmup, self.total = lr, warmup_updates, total_num_update
        self.end_lr, self.power = end_learning_rate, power

    def lr_for(self, num_updates_done: int) -> float:
        if self.warmup > 0 and num_updates_done == 0:
            return self.base_lr / self.warmup
        return polynomial_decay_lr(num_updates_done, self.base_lr, self.warmup, self.total, self.end_lr, self.power)

    def state_dict(self):
        return {"base_lr": self.base_lr, "warmup": self.warmup, "total": self.total, "end_lr": self.end_lr,
                "power": self.power}

    def load_state_dict(self, sd):
        self.__dict__.update({k: sd[k] for k in ("base_lr", "warmup", "total", "end_lr", "power") if k in sd})
