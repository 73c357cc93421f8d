"""Weight initialisers of the reference (yoco/models/decoder/model_parallel_init.py:6-16).

Each is applied per logical weight (per q/k/v/g/gt block of a merged projection), so the fan-in/fan-out of xavier and
kaiming match the reference's separate ``Linear`` weights.
"""
import math

import torch
import torch.nn as nn


def init_method(t: torch.Tensor):
    nn.init.kaiming_uniform_(t, a=math.sqrt(5))


def qkvg_init_method(t: torch.Tensor):
    nn.init.xavier_uniform_(t, gain=2 ** -2.5)


def out_init_method(t: torch.Tensor):
    nn.init.xavier_uniform_(t, gain=2 ** -1)


def vocab_init_method(t: torch.Tensor):
    nn.init.normal_(t, mean=0, std=t.shape[1] ** -0.5)


def normal_init(std: float):
    def f(t: torch.Tensor):
        nn.init.normal_(t, mean=0.0, std=std)
    return f
