"""Per-device scratch buffers shared by the kernels.

* ``gemm_workspace``: fp32 split-K partial tiles (sized for one persistent wave
  of 148 CTAs x 128 x 256 fp32 accumulators),
* ``gemm_counters``: per-tile arrival counters; each split-K GEMM leaves them
  at zero when it finishes,
* ``status``: one int32 word that bounded device-side waits write an error code
  into instead of hanging.  :func:`check_status` turns it into an exception.
"""

from __future__ import annotations

import threading

import torch

_lock = threading.Lock()
_buffers: dict[tuple[int, str], torch.Tensor] = {}

GEMM_WORKSPACE_FLOATS = 148 * 128 * 256
GEMM_COUNTER_SLOTS = 4096

ERROR_NAMES = {
    1: "TMA producer timed out waiting for a free shared-memory stage",
    2: "MMA issuer timed out waiting for a TMA tile",
    3: "epilogue timed out waiting for an accumulator",
    4: "MMA issuer timed out waiting for a free accumulator",
    5: "fused collective timed out waiting for a peer",
    6: "kernel rejected its arguments",
    7: "an index input (token id or KV slot) was out of range; the access was skipped",
}


def _get(device: torch.device, name: str, factory) -> torch.Tensor:
    index = device.index if device.index is not None else torch.cuda.current_device()
    key = (index, name)
    buffer = _buffers.get(key)
    if buffer is None:
        with _lock:
            buffer = _buffers.get(key)
            if buffer is None:
                buffer = factory(torch.device("cuda", index))
                _buffers[key] = buffer
    return buffer


def gemm_workspace(device: torch.device) -> torch.Tensor:
    return _get(device, "gemm_ws", lambda d: torch.empty(GEMM_WORKSPACE_FLOATS, dtype=torch.float32, device=d))


def gemm_counters(device: torch.device) -> torch.Tensor:
    return _get(device, "gemm_cnt", lambda d: torch.zeros(GEMM_COUNTER_SLOTS, dtype=torch.int32, device=d))


SAMPLER_SPLIT_ROWS = 4096   # csrc/sampling.h kGumbelSplitRows


def sampler_split(device: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-row scratch of the split-row Gumbel sampler (best key, arrival count), zero at rest."""
    best = _get(device, "gumbel_best", lambda d: torch.zeros(SAMPLER_SPLIT_ROWS, dtype=torch.int64, device=d))
    count = _get(device, "gumbel_count", lambda d: torch.zeros(SAMPLER_SPLIT_ROWS, dtype=torch.int32, device=d))
    return best, count


ROW_STATS_SPLIT_ROWS, ROW_STATS_MAX_SPLIT = 4096, 16   # csrc/sampling.h


def row_stats_split(device: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
    """Scratch of the split-row statistics kernel: per-chunk partials and per-row arrival counts
    (the counts are zero at rest)."""
    part = _get(device, "rowstats_part",
                lambda d: torch.zeros(ROW_STATS_SPLIT_ROWS * ROW_STATS_MAX_SPLIT * 3, dtype=torch.float32, device=d))
    count = _get(device, "rowstats_count", lambda d: torch.zeros(ROW_STATS_SPLIT_ROWS, dtype=torch.int32, device=d))
    return part, count


def scratch(device: torch.device, name: str, numel: int, dtype: torch.dtype) -> torch.Tensor:
    """A named per-device scratch buffer of at least ``numel`` elements (grown on demand).

    The buffer is reused across calls on the same stream, so a caller must be done
    with one use before the next call of the same name.
    """
    index = device.index if device.index is not None else torch.cuda.current_device()
    key = (index, "scratch:" + name)
    with _lock:
        buffer = _buffers.get(key)
        if buffer is None or buffer.numel() < numel or buffer.dtype != dtype:
            buffer = torch.empty(numel, dtype=dtype, device=torch.device("cuda", index))
            _buffers[key] = buffer
    return buffer[:numel]


def zeros(device: torch.device, name: str, numel: int, dtype: torch.dtype) -> torch.Tensor:
    """A named per-device buffer created zeroed once (for counters that kernels reset themselves)."""
    return _get(device, "zeros:" + name, lambda d: torch.zeros(numel, dtype=dtype, device=d))


def status(device: torch.device) -> torch.Tensor:
    return _get(device, "status", lambda d: torch.zeros(1, dtype=torch.int32, device=d))


def check_status(device: torch.device | None = None) -> None:
    """Raise if any bounded device wait on ``device`` gave up (synchronises)."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    word = status(device)
    code = int(word.item())
    if code:
        word.zero_()
        raise RuntimeError(f"device kernel error {code}: {ERROR_NAMES.get(code, 'unknown')}")
