"""CUDA-event timing helpers plus an L2 flush.

The public names and signatures (``measure_us``, ``percentile``,
``summarize``) are those of the reference's
``python/cuda_operator_lab/benchmarking.py:11-72``, so benchmark scripts
written against it keep working; the implementations are this library's own:

* ``measure_us`` keeps one event pair per sample and reads all elapsed times
  after the loop.  Each sample starts on an idle stream (the stream is drained
  after every sample), and ``before_each`` -- e.g. an :class:`L2Flusher` -- is
  enqueued ahead of the start event, so cache preparation never falls inside a
  timed interval.
* ``percentile`` / ``summarize`` use the inclusive linear-interpolation
  quantile (``torch.quantile``, float64) over the samples.
"""

from __future__ import annotations

import statistics
from collections.abc import Callable, Sequence

import torch


def _check_counts(warmup: int, repeats: int) -> None:
    if warmup < 0:
        raise ValueError("warmup must be non-negative")
    if repeats <= 0:
        raise ValueError("repeats must be positive")


def measure_us(
    fn: Callable[[], object],
    *,
    warmup: int,
    repeats: int,
    before_each: Callable[[], object] | None = None,
) -> list[float]:
    """Device time of each of `repeats` isolated calls of `fn`, in microseconds."""
    _check_counts(warmup, repeats)
    prepare = before_each if before_each is not None else (lambda: None)
    for _ in range(warmup):
        prepare()
        fn()
    stream = torch.cuda.current_stream()
    stream.synchronize()
    pairs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
             for _ in range(repeats)]
    for begin, finish in pairs:
        prepare()
        begin.record(stream)
        fn()
        finish.record(stream)
        stream.synchronize()  # the next sample starts on an idle GPU
    return [1000.0 * begin.elapsed_time(finish) for begin, finish in pairs]


def _quantiles(samples: Sequence[float], qs: Sequence[float]) -> list[float]:
    if len(samples) == 0:
        raise ValueError("samples must not be empty")
    if any(not 0.0 <= q <= 1.0 for q in qs):
        raise ValueError("q must be in [0, 1]")
    values = torch.tensor(list(samples), dtype=torch.float64)
    points = torch.tensor(list(qs), dtype=torch.float64)
    return torch.quantile(values, points, interpolation="linear").tolist()


def percentile(samples: list[float], q: float) -> float:
    """Inclusive linearly interpolated quantile of `samples`, q in [0, 1]."""
    return _quantiles(samples, [q])[0]


def summarize(samples: list[float]) -> tuple[float, float, float]:
    """(median, P50, P95) of per-call times in microseconds."""
    p50, p95 = _quantiles(samples, [0.50, 0.95])
    return statistics.median(samples), p50, p95


def measure_batch_us(fn: Callable[[], object], *, warmup: int, repeats: int) -> float:
    """Average device time per call of `repeats` back-to-back calls between
    one event pair: the steady-state cost when the GPU never idles (host
    launch overhead is hidden unless the host is slower than the kernels)."""
    _check_counts(warmup, repeats)
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
