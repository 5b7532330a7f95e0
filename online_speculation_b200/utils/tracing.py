"""Named trace ranges for the timeline tools: NVTX on the GPU and ``torch.profiler`` scopes.

``trace_range("engine.sample_batch")`` opens an NVTX range (visible to ncu / Nsight) and a
``record_function`` scope (visible in ``torch.profiler`` traces) around a host-side phase; the
ranges cost a few microseconds, so they wrap calls, not kernels.  ``set_tracing(False)`` turns
them into no-ops.  The blockspec profile mode's scope names (``blockspec.sample_ar`` and the
like) follow the reference's; the engine and trainer phases are this package's.
"""

from __future__ import annotations

import contextlib
from collections.abc import Iterator

import torch

_enabled = True


def set_tracing(on: bool) -> None:
    global _enabled
    _enabled = bool(on)


def tracing_enabled() -> bool:
    return _enabled


@contextlib.contextmanager
def trace_range(name: str) -> Iterator[None]:
    if not _enabled:
        yield
        return
    nvtx = torch.cuda.is_available()
    if nvtx:
        torch.cuda.nvtx.range_push(name)
    try:
        with torch.autograd.profiler.record_function(name):
            yield
    finally:
        if nvtx:
            torch.cuda.nvtx.range_pop()
