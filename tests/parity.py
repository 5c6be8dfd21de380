"""Helpers for the GPU parity tests: run the oracle on the CPU on (a sample
of) the same inputs and gate the native output with the reference's metric."""

from __future__ import annotations

import numpy as np
import torch

from kernelo_b200.testing import verify


def host(t: torch.Tensor) -> np.ndarray:
    """Exact values of a (low-precision) tensor as float64 on the host."""
    return t.detach().to("cpu", torch.float64).numpy()


def gate(expected: np.ndarray, out: torch.Tensor, dtype: torch.dtype, *, context: str = "",
         threshold: float | None = None):
    result = verify(torch.from_numpy(np.asarray(expected, dtype=np.float64)), out.detach().cpu().double(),
                    dtype=dtype, threshold=threshold)
    assert result.passed, f"{context}: {result.reason}"
    return result


def sample_rows(m: int, count: int = 64, seed: int = 0) -> np.ndarray:
    """Row indices for a sampled check at full size: first, last and random rows."""
    if m <= count:
        return np.arange(m)
    rng = np.random.default_rng(seed)
    picked = set(rng.choice(m, size=count - 2, replace=False).tolist()) | {0, m - 1}
    return np.array(sorted(picked))
