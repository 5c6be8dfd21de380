"""KernelForge-B200: the KernelForge kernel hot path, native to B200 (sm_100a).

The public names match ``kernelforge/__init__.py``. Importing the package
touches neither CUDA nor the native library; kernels are reached through
:func:`get_operator` or the wrappers in :mod:`kernelo_b200.kernels`, and the
library ``libkernelo_b200.so`` is loaded on the first kernel call.
"""

from __future__ import annotations

from kernelo_b200.benchmark.runner import TimingResult, benchmark
from kernelo_b200.kernels import get_operator, operator_names
from kernelo_b200.runtime.env import DeviceCaps, Environment, capture_environment, device_caps
from kernelo_b200.testing import VerificationResult, verify
from kernelo_b200.tuning.config import KernelConfig, Problem
from kernelo_b200.tuning.tuner import Tuner, TuningResult

__version__ = "0.1.0"

__all__ = [
    "DeviceCaps",
    "Environment",
    "KernelConfig",
    "Problem",
    "TimingResult",
    "Tuner",
    "TuningResult",
    "VerificationResult",
    "__version__",
    "benchmark",
    "capture_environment",
    "device_caps",
    "get_operator",
    "operator_names",
    "verify",
]
