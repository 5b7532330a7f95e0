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


class _Counted:
    """Proxy that counts every kernel launch made through the extension."""

    def __init__(self, mod):
        self._mod = mod
        self.launches = 0

    def __getattr__(self, name):
        attr = getattr(self._mod, name)
        if callable(attr) and not isinstance(attr, type) and name not in ("gemm_pick_bn",):
            def call(*args, **kwargs):
                self.launches += 1
                return attr(*args, **kwargs)
            return call
        return attr


_counted = None


def launches() -> int:
    """Kernel launches issued through the extension so far (graph replays not included)."""
    return 0 if _counted is None else _counted.launches


def require():
    global _counted
    ext = load()
    if ext is not None and _counted is None:
        _counted = _Counted(ext)
    if ext is None:
        raise RuntimeError(
            "the online_speculation_b200 CUDA extension is not built; run "
            "`python setup.py build_ext --inplace` (sm_100a) before using CUDA tensors"
        ) from _error
    return _counted
