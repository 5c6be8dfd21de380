"""Kernel-launch accounting with torch.profiler (``kernelforge/profiling/pytorch_profiler.py``).

Counts the device kernels one call launches (the fusion claim: one launch for
the fused linear against three or more unfused) and their device time. CUPTI
sees launches from the native library like any other, so the counts include
``libkernelo_b200`` kernels.
"""

from __future__ import annotations

from collections import Counter
from collections.abc import Callable
from dataclasses import dataclass, field

import torch


@dataclass(frozen=True)
class KernelProfile:
    label: str
    iterations: int
    kernel_launches: int
    device_time_us: float
    kernels: dict[str, int] = field(default_factory=dict)

    @property
    def launches_per_iteration(self) -> float:
        return self.kernel_launches / self.iterations

    @property
    def device_time_per_iteration_us(self) -> float:
        return self.device_time_us / self.iterations


def _is_kernel(name: str) -> bool:
    lowered = name.lower()
    return not (lowered.startswith("memcpy") or lowered.startswith("memset") or "cudaevent" in lowered)


def profile_kernels(fn: Callable[[], object], *, label: str, warmup: int = 5,
                    iterations: int = 10) -> KernelProfile:
    if not torch.cuda.is_available():
        raise RuntimeError("profile_kernels needs a CUDA device")
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(iterations):
            fn()
        torch.cuda.synchronize()
    names: Counter[str] = Counter()
    device_us = 0.0
    for evt in prof.events():
        if evt.device_type == torch.autograd.DeviceType.CUDA and _is_kernel(evt.name):
            names[evt.name] += 1
            device_us += evt.device_time_total if hasattr(evt, "device_time_total") else evt.cuda_time_total
    return KernelProfile(label, iterations, sum(names.values()), device_us, dict(names))
