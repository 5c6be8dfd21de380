"""Timing harness: device time of one call, as a distribution.

The reference's ``benchmark`` (``kernelforge/benchmark/runner.py:123-207``)
fixes the method this keeps: warm-up calls, then per-iteration CUDA events on
the current stream with a single synchronisation after the loop (so no sync
leaks into a sample), the L2 emptied before every timed iteration, and the
samples summarised as median / p95 / p99 with the median used for ranking.

Here a timer is a small strategy object -- :class:`_EventClock` on a CUDA
device, :class:`_HostClock` without one -- that turns a callable into a list
of per-iteration milliseconds; :func:`benchmark` picks one and
:meth:`TimingResult.from_samples` summarises. A host-clock result is labelled
``perf_counter`` so it can never pass for device time.

Beyond the reference: the L2 is emptied by writing a buffer twice its size
and then reading another (clean lines, no write-back debt for the timed
kernel), and :func:`graph_time_per_launch` times back-to-back launches
replayed as one CUDA graph over rotating input sets.
"""

from __future__ import annotations

import time
from collections.abc import Callable
from dataclasses import dataclass, field

import numpy as np
import torch

from kernelo_b200.runtime.env import device_caps

DEFAULT_WARMUP = 25
DEFAULT_ITERATIONS = 200

#: CUDA event resolution is about half a microsecond; medians at or below this
#: are reported but not comparable.
TIMER_RESOLUTION_MS = 0.002


@dataclass(frozen=True)
class TimingResult:
    """Milliseconds per call: the summary statistics of one timing run."""

    median_ms: float
    mean_ms: float
    std_ms: float
    min_ms: float
    max_ms: float
    p95_ms: float
    p99_ms: float
    warmup: int
    iterations: int
    timer: str
    flushed_l2: bool
    samples_ms: tuple[float, ...] = field(default=(), repr=False)

    @classmethod
    def from_samples(cls, samples_ms, *, warmup: int, iterations: int, timer: str, flushed_l2: bool,
                     keep_samples: bool = False) -> TimingResult:
        values = np.sort(np.fromiter((float(v) for v in samples_ms), dtype=np.float64))
        if values.size == 0:
            raise ValueError("cannot summarize an empty set of timing samples")
        median, p95, p99 = np.quantile(values, (0.5, 0.95, 0.99))
        spread = float(np.std(values, ddof=1)) if values.size > 1 else 0.0
        kept = tuple(float(v) for v in samples_ms) if keep_samples else ()
        return cls(float(median), float(values.mean()), spread, float(values[0]), float(values[-1]),
                   float(p95), float(p99), warmup, iterations, timer, flushed_l2, kept)

    @property
    def at_timer_resolution(self) -> bool:
        return self.timer == "cuda_event" and self.median_ms <= TIMER_RESOLUTION_MS

    @property
    def median_us(self) -> float:
        return 1e3 * self.median_ms

    def as_dict(self) -> dict[str, float | int | str | bool]:
        names = ("median_ms", "mean_ms", "std_ms", "min_ms", "max_ms", "p95_ms", "p99_ms", "warmup", "iterations",
                 "timer", "flushed_l2")
        return {name: getattr(self, name) for name in names}


def summarize(
    samples_ms,
    *,
    warmup: int,
    iterations: int,
    timer: str,
    flushed_l2: bool,
    keep_samples: bool = False,
) -> TimingResult:
    """Distribution of per-iteration times (linear-interpolated percentiles)."""
    return TimingResult.from_samples(samples_ms, warmup=warmup, iterations=iterations, timer=timer,
                                     flushed_l2=flushed_l2, keep_samples=keep_samples)


def l2_flush_buffer(device: torch.device) -> torch.Tensor:
    """A byte buffer twice the size of the device's L2."""
    return torch.empty(2 * device_caps(device).l2_cache_bytes, dtype=torch.int8, device=device)


class L2Flush:
    """Evicts the next kernel's inputs from L2 and leaves L2 holding clean lines.

    Writing a buffer twice the L2 size pushes every earlier line out. Those
    written lines are dirty, and a kernel that ran next would pay for writing
    them back -- up to 126 MB of extra DRAM traffic, which halves the apparent
    bandwidth of a kernel whose working set is about the size of L2 (a decode
    GEMV's 90 MB weight). So a second buffer of the same size is then read,
    which replaces the dirty lines with clean ones. Finally the stream sleeps
    for ``guard_cycles`` so that the host has queued the timed launches before
    the start event fires: the timed region then holds device time only.
    """

    def __init__(self, device: torch.device, *, guard_cycles: int = 200_000) -> None:
        self.write_buf = l2_flush_buffer(device)
        self.read_buf = l2_flush_buffer(device)
        self.guard_cycles = guard_cycles

    def __call__(self) -> None:
        self.write_buf.zero_()
        self.read_buf.max()
        sleep = getattr(torch.cuda, "_sleep", None)
        if sleep is not None and self.guard_cycles > 0:
            sleep(self.guard_cycles)


class _HostClock:
    """Wall-clock timing for CPU callables (no device to synchronise)."""

    name = "perf_counter"
    flushes = False

    def samples(self, fn: Callable[[], object], iterations: int) -> list[float]:
        out = []
        for _ in range(iterations):
            t0 = time.perf_counter()
            fn()
            out.append(1e3 * (time.perf_counter() - t0))
        return out


class _EventClock:
    """CUDA events around each call on the current stream; one sync at the end.
    With ``flush``, the L2 is emptied before each start event (outside the
    measured interval: the stream is in order)."""

    name = "cuda_event"

    def __init__(self, device: torch.device, flush: bool) -> None:
        self.device = device
        self.flushes = flush
        self._flush = L2Flush(device) if flush else None

    def samples(self, fn: Callable[[], object], iterations: int) -> list[float]:
        torch.cuda.synchronize(self.device)
        marks = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                 for _ in range(iterations)]
        for begin, finish in marks:
            if self._flush is not None:
                self._flush()
            begin.record()
            fn()
            finish.record()
        torch.cuda.synchronize(self.device)
        return [begin.elapsed_time(finish) for begin, finish in marks]


def benchmark(
    fn: Callable[[], object],
    *,
    warmup: int = DEFAULT_WARMUP,
    iterations: int = DEFAULT_ITERATIONS,
    device: torch.device | str | None = None,
    flush_l2: bool = True,
    keep_samples: bool = False,
) -> TimingResult:
    """Time the zero-argument callable ``fn`` and summarise the samples."""
    if warmup < 0:
        raise ValueError(f"warmup must be non-negative, got {warmup}")
    if iterations < 1:
        raise ValueError(f"iterations must be at least 1, got {iterations}")
    target = torch.device(device) if device is not None else None
    if torch.cuda.is_available() and (target is None or target.type == "cuda"):
        if target is None or target.index is None:
            target = torch.device("cuda", torch.cuda.current_device())
        clock: _HostClock | _EventClock = _EventClock(target, flush_l2)
    else:
        clock = _HostClock()
    for _ in range(warmup):
        fn()
    samples = clock.samples(fn, iterations)
    return TimingResult.from_samples(samples, warmup=warmup, iterations=iterations, timer=clock.name,
                                     flushed_l2=clock.flushes, keep_samples=keep_samples)


def cross_check_median_ms(
    fn: Callable[[], object], *, warmup: int = DEFAULT_WARMUP, min_run_time: float = 1.0
) -> float:
    """A second opinion on :func:`benchmark`: the median that
    ``torch.utils.benchmark`` measures for ``fn`` (its own adaptive loop,
    host-side timing around synchronised blocks), in milliseconds."""
    from torch.utils.benchmark import Timer

    for _ in range(warmup):
        fn()
    measurement = Timer(stmt="fn()", globals={"fn": fn}).blocked_autorange(min_run_time=min_run_time)
    return 1e3 * float(measurement.median)


def rotation_sets(bytes_per_set: int, device: torch.device | str | None = None, *, minimum: int = 2) -> int:
    """Input sets to cycle through so that the sets together exceed twice the L2."""
    gpu = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    l2 = device_caps(gpu).l2_cache_bytes
    return max(minimum, -(-2 * l2 // max(1, bytes_per_set)) + 1)


def graph_time_per_launch(calls: list[Callable[[], object]], *, replays: int = 5) -> float:
    """Median device milliseconds per launch of ``calls`` replayed as one CUDA graph.

    ``calls`` should cycle through input sets whose total exceeds the L2 (see
    :func:`rotation_sets`), so that no launch finds its inputs cached. The
    graph replays the launches back to back: host overhead and the per-event
    launch gap (about 6 us on B200) stay out of the per-launch figure.
    """
    if not calls:
        raise ValueError("no calls to time")
    for call in calls:  # allocations, kernel attributes, workspaces
        call()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for call in calls:
            call()
    graph.replay()
    torch.cuda.synchronize()
    samples = []
    for _ in range(replays):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        graph.replay()
        end.record()
        end.synchronize()
        samples.append(start.elapsed_time(end) / len(calls))
    del graph
    samples.sort()
    return samples[len(samples) // 2]
