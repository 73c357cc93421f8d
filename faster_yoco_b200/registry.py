"""Name registries for models, tasks and criterions (the fairseq-style ``--arch`` / ``--task`` / ``--criterion``
lookup of the reference; yoco/models/__init__.py:20-41, tasks/__init__.py:10-32, criterions/__init__.py:4-8).

Registration happens at import of :mod:`faster_yoco_b200.registry_all`, which imports every built-in module; unlike
the reference, importing a module here installs no monkey-patches anywhere.
"""
from __future__ import annotations

from typing import Callable, Dict

MODELS: Dict[str, Callable] = {}
TASKS: Dict[str, Callable] = {}
CRITERIONS: Dict[str, Callable] = {}


def _reg(table: Dict[str, Callable], kind: str):
    def outer(name: str):
        def deco(obj):
            if name in table and table[name] is not obj:
                raise ValueError(f"{kind} {name!r} registered twice")
            table[name] = obj
            return obj
        return deco
    return outer


register_model = _reg(MODELS, "model")
register_task = _reg(TASKS, "task")
register_criterion = _reg(CRITERIONS, "criterion")


def get(table: Dict[str, Callable], name: str, kind: str):
    import faster_yoco_b200.registry_all  # noqa: F401  (populates the tables)
    if name not in table:
        raise KeyError(f"unknown {kind} {name!r}; registered: {sorted(table)}")
    return table[name]


def get_model(name):
    return get(MODELS, name, "model")


def get_task(name):
    return get(TASKS, name, "task")


def get_criterion(name):
    return get(CRITERIONS, name, "criterion")
