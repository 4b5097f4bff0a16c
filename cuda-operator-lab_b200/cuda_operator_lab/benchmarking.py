"""CUDA-event timing helpers (same API as the reference's
``python/cuda_operator_lab/benchmarking.py:11-72``) plus an L2 flush.

``measure_us`` enqueues ``before_each`` (for example :func:`l2_flush`) on the
current stream ahead of the start event, so cache preparation is never inside
the timed interval.
"""

from __future__ import annotations

import statistics
from collections.abc import Callable

import torch


def measure_us(
    fn: Callable[[], object],
    *,
    warmup: int,
    repeats: int,
    before_each: Callable[[], object] | None = None,
) -> list[float]:
    """Per-call device time in microseconds, one CUDA-event pair per call."""
    if warmup < 0:
        raise ValueError("warmup must be non-negative")
    if repeats <= 0:
        raise ValueError("repeats must be positive")
    for _ in range(warmup):
        if before_each is not None:
            before_each()
        fn()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    samples: list[float] = []
    for _ in range(repeats):
        if before_each is not None:
            before_each()
        start.record()
        fn()
        end.record()
        end.synchronize()
        samples.append(start.elapsed_time(end) * 1000.0)
    return samples


def percentile(samples: list[float], q: float) -> float:
    """Linear-interpolation percentile, q in [0, 1]."""
    if not samples:
        raise ValueError("samples must not be empty")
    if not 0.0 <= q <= 1.0:
        raise ValueError("q must be in [0, 1]")
    ordered = sorted(samples)
    if len(ordered) == 1:
        return ordered[0]
    position = (len(ordered) - 1) * q
    lower = int(position)
    upper = min(lower + 1, len(ordered) - 1)
    weight = position - lower
    return ordered[lower] * (1.0 - weight) + ordered[upper] * weight


def summarize(samples: list[float]) -> tuple[float, float, float]:
    """(median, P50, P95) in microseconds."""
    return statistics.median(samples), percentile(samples, 0.50), percentile(samples, 0.95)


def measure_batch_us(fn: Callable[[], object], *, warmup: int, repeats: int) -> float:
    """Average device time per call of `repeats` back-to-back calls between
    one event pair: the steady-state cost when the GPU never idles (host
    launch overhead is hidden unless the host is slower than the kernels)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(repeats):
        fn()
    end.record()
    end.synchronize()
    return start.elapsed_time(end) * 1000.0 / repeats


class L2Flusher:
    """Evicts the L2 between samples by reading a buffer of twice its size.

    Reading (not writing) leaves the L2 full of clean lines, so the measured
    kernel pays only for its own DRAM traffic, not for writing back the
    flush buffer's dirty lines.
    """

    def __init__(self, device: torch.device | int | None = None) -> None:
        props = torch.cuda.get_device_properties(device if device is not None else 0)
        size = max(2 * int(getattr(props, "L2_cache_size", 0) or 0), 256 << 20)
        dev = device if device is not None else "cuda"
        self.buffer = torch.ones(size // 4, dtype=torch.float32, device=dev)
        self.sink = torch.empty((), dtype=torch.float32, device=dev)

    def __call__(self) -> None:
        torch.sum(self.buffer, dim=0, out=self.sink)
