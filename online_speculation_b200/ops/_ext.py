"""Loader for the compiled sm_100a extension (``online_speculation_b200._C``).

CUDA tensors always go through the compiled kernels.  When the extension is
missing on a machine with a GPU, :func:`require` raises instead of silently
falling back to PyTorch; CPU tensors use the PyTorch oracle implementations of
each op, which the tests compare the kernels against.
"""

from __future__ import annotations

import importlib

_ext = None
_error: Exception | None = None


def load():
    global _ext, _error
    if _ext is None and _error is None:
        try:
            _ext = importlib.import_module("online_speculation_b200._C")
        except ImportError as error:  # pragma: no cover - depends on the build
            _error = error
    return _ext


def available() -> bool:
    return load() is not None


def require():
    ext = load()
    if ext is None:
        raise RuntimeError(
            "the online_speculation_b200 CUDA extension is not built; run "
            "`python setup.py build_ext --inplace` (sm_100a) before using CUDA tensors"
        ) from _error
    return ext
