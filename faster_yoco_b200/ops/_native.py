"""Loader for the in-tree sm_100a extension (``faster_yoco_b200/_C*.so``).

On a machine with a CUDA device the extension is required: every native op raises ``NativeUnavailable`` with the
import error instead of silently running a PyTorch fallback. On CPU-only machines the model runs the reference
PyTorch expressions and the extension is never touched.
"""
from __future__ import annotations

import importlib

_C = None
_ERR = None


class NativeUnavailable(RuntimeError):
    pass


def load():
    global _C, _ERR
    if _C is not None or _ERR is not None:
        return _C
    try:
        import torch  # noqa: F401  (the extension links against libtorch)
        _C = importlib.import_module("faster_yoco_b200._C")
    except Exception as e:  # pragma: no cover - depends on the build
        _ERR = e
        _C = None
    return _C


def lib():
    """The extension module, or raise with the reason it is missing."""
    m = load()
    if m is None:
        raise NativeUnavailable(
            "faster_yoco_b200._C is not built or failed to load (%r). Build it with "
            "`python -c 'import __graft_entry__ as g; g.build()'` or `python setup.py build_ext --inplace`." % (_ERR,))
    return m


def available() -> bool:
    return load() is not None


def so_path():
    m = load()
    return getattr(m, "__file__", None) if m is not None else None


def has(name: str) -> bool:
    m = load()
    return m is not None and hasattr(m, name)

