"""Named shape suites (``kernelforge/benchmark/workloads.py:39-136``).

``smoke``, ``sweep``, ``transformer`` and ``correctness`` keep the reference's
shapes so results stay comparable with it; ``baseline`` adds the shapes this
project is measured on (the fused linear 4096x11008x4096, decode GEMMs at
M in {1,4,16}, softmax over [32768, C] and RMSNorm over [16384, 4096/8192])
and ``sweep_sm100`` the tuner-sweep shapes (primes, one-off-a-tile, M=1).
"""

from __future__ import annotations

import torch

from kernelo_b200.tuning.config import Problem

# Llama-2-7B geometry: hidden 4096, MLP intermediate 11008.
HIDDEN = 4096
INTERMEDIATE = 11008
TOKEN_COUNTS = (1, 32, 512, 2048)

_MATMUL: dict[str, tuple[tuple[int, int, int], ...]] = {
    "smoke": ((512, 512, 512), (1024, 1024, 1024)),
    "sweep": (
        (512, 512, 512),
        (1024, 1024, 1024),
        (2048, 2048, 2048),
        (4096, 4096, 4096),
        (512, 4096, 4096),
        (4096, 512, 4096),
        (4096, 4096, 512),
        (2048, 4096, 4096),
        (1024, 4096, 1024),
        (4096, 1024, 4096),
    ),
    "transformer": tuple(
        shape
        for t in TOKEN_COUNTS
        for shape in ((t, HIDDEN, HIDDEN), (t, INTERMEDIATE, HIDDEN), (t, HIDDEN, INTERMEDIATE))
    ),
    "correctness": (
        (1, 1, 1),
        (1, 128, 128),
        (128, 1, 128),
        (128, 128, 1),
        (127, 127, 127),
        (128, 128, 128),
        (129, 129, 129),
        (257, 129, 65),
        (511, 769, 1025),
        (1023, 1023, 1023),
        (1024, 1024, 1024),
        (2057, 127, 513),
        (768, 2048, 4096),
    ),
    "baseline": (
        (2048, 4096, 4096),
        (4096, INTERMEDIATE, HIDDEN),
        (1, INTERMEDIATE, HIDDEN),
        (4, INTERMEDIATE, HIDDEN),
        (16, INTERMEDIATE, HIDDEN),
    ),
    "sweep_sm100": (
        (4099, 4099, 4099),
        (1021, 2053, 509),
        (129, 129, 129),
        (257, 257, 257),
        (1, INTERMEDIATE, HIDDEN),
        (2048, 4096, 4096),
    ),
}

_ROWS: dict[str, tuple[tuple[int, int], ...]] = {
    "smoke": ((2048, 1024), (4096, 4096)),
    "sweep": tuple(
        (r, c) for r in (512, 2048, 8192) for c in (128, 256, 512, 1024, 2048, 4096, 8192)
    ),
    "transformer": tuple((t, HIDDEN) for t in TOKEN_COUNTS) + tuple((t, 768) for t in TOKEN_COUNTS),
    "correctness": (
        (1, 1),
        (1, 4096),
        (3, 127),
        (17, 257),
        (128, 511),
        (333, 769),
        (1024, 1023),
        (2048, 1024),
        (4096, 4096),
        (129, 8192),
    ),
    "baseline_softmax": ((32768, 1000), (32768, 4096), (32768, 4097), (32768, 32000)),
    "baseline_rmsnorm": ((16384, 4096), (16384, 8192)),
}

#: Decode shapes (M rows of x, N, K) for the GEMV's smoke and sweep suites.
_GEMV: dict[str, tuple[tuple[int, int, int], ...]] = {
    "smoke": ((1, 4096, 4096), (4, 4096, 4096)),
    "sweep": ((1, 4096, 4096), (1, 11008, 4096), (4, 11008, 4096), (16, 11008, 4096), (16, 4096, 11008),
              (64, 11008, 4096)),
}

SUITES: tuple[str, ...] = ("smoke", "sweep", "transformer", "correctness", "baseline", "sweep_sm100")


def problems(operation: str, suite: str = "sweep", dtype: str | torch.dtype = "fp16") -> list[Problem]:
    """Every problem of ``suite`` for ``operation``."""
    if suite not in SUITES:
        raise ValueError(f"unknown suite {suite!r}; available: {', '.join(SUITES)}")
    if operation in ("matmul", "fused_linear", "gemv"):
        shapes = _MATMUL[suite]
        if operation == "gemv":
            # The GEMM suites' smoke and sweep shapes are all prefill-sized:
            # the decode GEMV gets decode shapes of its own there.
            shapes = _GEMV.get(suite) or tuple(s for s in shapes if s[0] <= 256)
        return [Problem.create(operation, dtype, M=m, N=n, K=k) for m, n, k in shapes]
    if operation in ("softmax", "rmsnorm"):
        key = suite
        if suite == "baseline":
            key = f"baseline_{operation}"
        elif suite == "sweep_sm100":
            key = "correctness"
        return [Problem.create(operation, dtype, rows=r, cols=c) for r, c in _ROWS[key]]
    raise ValueError(f"no workload suite defined for {operation!r}")
