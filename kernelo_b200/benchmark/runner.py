"""CUDA-event timing harness (``kernelforge/benchmark/runner.py:123-207``).

Each timed iteration is bracketed by a pair of CUDA events recorded on the
current stream; the stream is synchronised once after the loop, so no
per-iteration sync leaks into the samples. Before every iteration an
L2-sized buffer is zeroed (enqueued before the start event, so outside the
measured interval) to keep a previous iteration's operands from being served
out of the 126 MB L2. Results are summarised as a distribution (median, p95,
p99) and ranked on the median.

Without a CUDA device the harness falls back to ``time.perf_counter`` and
labels the result ``perf_counter`` so a CPU timing can never pass for a GPU one.
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

    @property
    def at_timer_resolution(self) -> bool:
        return self.timer == "cuda_event" and self.median_ms <= TIMER_RESOLUTION_MS

    @property
    def median_us(self) -> float:
        return self.median_ms * 1e3

    def as_dict(self) -> dict[str, float | int | str | bool]:
        return {
            "median_ms": self.median_ms,
            "mean_ms": self.mean_ms,
            "std_ms": self.std_ms,
            "min_ms": self.min_ms,
            "max_ms": self.max_ms,
            "p95_ms": self.p95_ms,
            "p99_ms": self.p99_ms,
            "warmup": self.warmup,
            "iterations": self.iterations,
            "timer": self.timer,
            "flushed_l2": self.flushed_l2,
        }


def summarize(
    samples_ms,
    *,
    warmup: int,
    iterations: int,
    timer: str,
    flushed_l2: bool,
    keep_samples: bool = False,
) -> TimingResult:
    """Distribution of per-iteration times (numpy's linear-interpolated percentiles)."""
    arr = np.asarray(list(samples_ms), dtype=np.float64)
    if arr.size == 0:
        raise ValueError("cannot summarize an empty set of timing samples")
    p95, p99 = np.percentile(arr, [95, 99])
    return TimingResult(
        median_ms=float(np.median(arr)),
        mean_ms=float(arr.mean()),
        std_ms=float(arr.std(ddof=1)) if arr.size > 1 else 0.0,
        min_ms=float(arr.min()),
        max_ms=float(arr.max()),
        p95_ms=float(p95),
        p99_ms=float(p99),
        warmup=warmup,
        iterations=iterations,
        timer=timer,
        flushed_l2=flushed_l2,
        samples_ms=tuple(float(x) for x in arr) if keep_samples else (),
    )


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
    on_gpu = torch.cuda.is_available() and (target is None or target.type == "cuda")

    for _ in range(warmup):
        fn()

    if not on_gpu:
        samples = []
        for _ in range(iterations):
            start = time.perf_counter()
            fn()
            samples.append((time.perf_counter() - start) * 1e3)
        return summarize(
            samples,
            warmup=warmup,
            iterations=iterations,
            timer="perf_counter",
            flushed_l2=False,
            keep_samples=keep_samples,
        )

    gpu = target if target is not None else torch.device("cuda", torch.cuda.current_device())
    torch.cuda.synchronize(gpu)
    flush = L2Flush(gpu) if flush_l2 else None
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(iterations)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(iterations)]
    for i in range(iterations):
        if flush is not None:
            flush()
        starts[i].record()
        fn()
        ends[i].record()
    torch.cuda.synchronize(gpu)
    return summarize(
        [s.elapsed_time(e) for s, e in zip(starts, ends)],
        warmup=warmup,
        iterations=iterations,
        timer="cuda_event",
        flushed_l2=flush_l2,
        keep_samples=keep_samples,
    )


def cross_check_median_ms(
    fn: Callable[[], object], *, warmup: int = DEFAULT_WARMUP, min_run_time: float = 1.0
) -> float:
    """Median latency from ``torch.utils.benchmark``: a second opinion on the loop above."""
    import torch.utils.benchmark as tbench

    for _ in range(warmup):
        fn()
    timer = tbench.Timer(stmt="fn()", globals={"fn": fn})
    return float(timer.blocked_autorange(min_run_time=min_run_time).median) * 1e3


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
