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
    kernel_time_us: dict[str, float] = field(default_factory=dict)

    @property
    def launches_per_iteration(self) -> float:
        return self.kernel_launches / self.iterations

    @property
    def device_time_per_iteration_us(self) -> float:
        return self.device_time_us / self.iterations

    def render(self, limit: int = 10) -> str:
        lines = [
            self.label,
            f"  kernel launches per call : {self.launches_per_iteration:.2f}",
            f"  device time per call     : {self.device_time_per_iteration_us:.1f} us",
        ]
        if self.kernels:
            lines.append("  kernels by device time:")
            ranked = sorted(self.kernels, key=lambda k: -self.kernel_time_us.get(k, 0.0))[:limit]
            width = min(62, max(len(k) for k in ranked))
            total = max(self.device_time_us, 1e-9)
            for name in ranked:
                t = self.kernel_time_us.get(name, 0.0)
                lines.append(f"    {name[:width]:<{width}}  {self.kernels[name] / self.iterations:>5.1f} launches  "
                             f"{t / self.iterations:>9.1f} us  {100 * t / total:>5.1f}%")
        return "\n".join(lines)


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
    from torch.profiler import ProfilerActivity, profile, schedule

    # One traced-but-discarded warm-up step first: a profiler session started
    # after an earlier one in the same process can miss the first launch it
    # sees, which would read as a fused call making fewer than one launch.
    with profile(activities=[ProfilerActivity.CUDA],
                 schedule=schedule(wait=0, warmup=1, active=iterations, repeat=1)) as prof:
        for step in range(iterations + 1):
            fn()
            if step == iterations:
                torch.cuda.synchronize()
            prof.step()
    names: Counter[str] = Counter()
    times: Counter[str] = Counter()
    for evt in prof.events():
        if evt.device_type == torch.autograd.DeviceType.CUDA and _is_kernel(evt.name):
            names[evt.name] += 1
            times[evt.name] += evt.device_time_total if hasattr(evt, "device_time_total") else evt.cuda_time_total
    return KernelProfile(label, iterations, sum(names.values()), float(sum(times.values())), dict(names),
                         dict(times))


def compare_launch_counts(candidates: dict[str, Callable[[], object]], *, warmup: int = 10,
                          iterations: int = 20) -> list[KernelProfile]:
    """Profile several implementations of one operation (``kernelforge/profiling/
    pytorch_profiler.py:137-149``): the fused linear's one launch against the
    unfused sequence's three, with device time per kernel."""
    return [profile_kernels(fn, label=label, warmup=warmup, iterations=iterations)
            for label, fn in candidates.items()]
