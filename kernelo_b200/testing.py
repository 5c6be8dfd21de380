"""The correctness gate (``kernelforge/testing.py:31-175``).

Nothing is ranked or benchmarked before it passes :func:`verify`. The metric is
scale invariant,

    err = max|out - ref| / max|ref|

with one threshold per dtype, so the same gate holds for a K=128 and a K=8192
GEMM whose outputs differ in magnitude by sqrt(K). The thresholds are the
reference's: fp32 1e-5 (which presumes an IEEE-fp32 reference, see
:func:`exact_fp32_matmul`), fp16 5e-3, bf16 2e-2.
"""

from __future__ import annotations

import contextlib
from dataclasses import dataclass

import torch

ERROR_THRESHOLDS: dict[torch.dtype, float] = {
    torch.float32: 1e-5,
    torch.float16: 5e-3,
    torch.bfloat16: 2e-2,
}


@dataclass(frozen=True)
class VerificationResult:
    passed: bool
    error: float
    max_abs_err: float
    mismatched: int
    total: int
    threshold: float
    reason: str = ""

    def __str__(self) -> str:
        if self.passed:
            return f"ok (err={self.error:.3e} <= {self.threshold:.1e})"
        return f"FAIL ({self.reason})"


def threshold_for(dtype: torch.dtype) -> float:
    if dtype not in ERROR_THRESHOLDS:
        known = sorted(str(d) for d in ERROR_THRESHOLDS)
        raise ValueError(f"no correctness threshold defined for {dtype}; known dtypes: {known}")
    return ERROR_THRESHOLDS[dtype]


def _fail(limit: float, total: int, bad: int, reason: str) -> VerificationResult:
    return VerificationResult(False, float("inf"), float("inf"), bad, total, limit, reason)


def verify(
    reference: torch.Tensor,
    output: torch.Tensor,
    *,
    dtype: torch.dtype | None = None,
    threshold: float | None = None,
) -> VerificationResult:
    """Compare ``output`` with ``reference`` under the dtype's threshold.

    ``dtype`` selects the threshold (default: the output's dtype). The
    comparison itself runs in fp32 so it is not subject to the format under
    test. A zero reference falls back to the absolute error.
    """
    limit = threshold if threshold is not None else threshold_for(
        dtype if dtype is not None else output.dtype
    )
    total = output.numel()
    if tuple(reference.shape) != tuple(output.shape):
        return _fail(
            limit,
            total,
            total,
            f"shape mismatch: reference {tuple(reference.shape)} vs output {tuple(output.shape)}",
        )
    if total == 0:
        return VerificationResult(True, 0.0, 0.0, 0, 0, limit)

    out = output.detach().to(device=reference.device, dtype=torch.float32)
    ref = reference.detach().to(torch.float32)
    finite = torch.isfinite(out)
    if not bool(finite.all()):
        bad = int((~finite).sum())
        return _fail(limit, total, bad, f"output contains {bad}/{total} non-finite values")

    diff = (out - ref).abs()
    max_abs = float(diff.max())
    scale = float(ref.abs().max())
    error = max_abs / scale if scale > 0 else max_abs
    budget = limit * scale if scale > 0 else limit
    mismatched = int((diff > budget).sum())
    passed = error <= limit
    reason = ""
    if not passed:
        reason = (
            f"normalised error {error:.3e} exceeds {limit:.1e} "
            f"(max|diff|={max_abs:.3e}, {mismatched}/{total} elements off)"
        )
    return VerificationResult(passed, error, max_abs, mismatched, total, limit, reason)


def assert_verified(
    reference: torch.Tensor,
    output: torch.Tensor,
    *,
    dtype: torch.dtype | None = None,
    threshold: float | None = None,
    context: str = "",
) -> VerificationResult:
    result = verify(reference, output, dtype=dtype, threshold=threshold)
    if not result.passed:
        raise AssertionError((f"{context}: " if context else "") + result.reason)
    return result


@contextlib.contextmanager
def exact_fp32_matmul():
    """Keep fp32 matmuls in IEEE fp32 (TF32 off) for the duration of the block.

    TF32 carries ~1e-3 relative error, a hundred times the fp32 gate, so any
    fp32 reference computed with it would be the least accurate number in the
    comparison. The previous settings are restored on exit, exception or not.
    """
    saved = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    try:
        yield
    finally:
        torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = saved
