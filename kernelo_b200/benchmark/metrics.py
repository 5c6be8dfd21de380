"""Algorithmic work models (``kernelforge/benchmark/metrics.py:17-88``).

Byte counts are the minimum traffic of a perfect kernel: every input read once,
every output written once. They are the ``roofline.achieved`` numerators; real
traffic (measured with ncu) above them is re-reading, which is what a fused or
better-tiled kernel removes.
"""

from __future__ import annotations


def matmul_flops(m: int, n: int, k: int) -> int:
    return 2 * m * n * k


def matmul_bytes(m: int, n: int, k: int, itemsize: int) -> int:
    """A read once, B read once, C written once."""
    return (m * k + k * n + m * n) * itemsize


def gemv_bytes(m: int, n: int, k: int, itemsize: int) -> int:
    """Decode-shape GEMM: X, W and Y each touched once (same model as matmul)."""
    return matmul_bytes(m, n, k, itemsize)


def elementwise_bytes(elements: int, itemsize: int, *, tensors: int) -> int:
    return elements * itemsize * tensors


def softmax_bytes(rows: int, cols: int, itemsize: int) -> int:
    """Read x, write y."""
    return 2 * rows * cols * itemsize


def rmsnorm_bytes(rows: int, cols: int, itemsize: int) -> int:
    """Read x, write y, read gamma once."""
    return (2 * rows * cols + cols) * itemsize


def fused_linear_bytes(m: int, n: int, k: int, itemsize: int, *, fused: bool) -> int:
    """``gelu(x @ w + b)``: operands once; output once fused, five times unfused
    (GEMM write, bias read+write, activation read+write)."""
    operands = m * k + k * n + n
    output = m * n if fused else 5 * m * n
    return (operands + output) * itemsize


def tflops(flops: int, ms: float) -> float:
    if ms <= 0:
        raise ValueError(f"latency must be positive, got {ms}")
    return flops / (ms * 1e-3) / 1e12


def gbps(num_bytes: int, ms: float) -> float:
    if ms <= 0:
        raise ValueError(f"latency must be positive, got {ms}")
    return num_bytes / (ms * 1e-3) / 1e9


def arithmetic_intensity(flops: int, num_bytes: int) -> float:
    if num_bytes <= 0:
        raise ValueError(f"byte count must be positive, got {num_bytes}")
    return flops / num_bytes


def speedup(baseline_ms: float, candidate_ms: float) -> float:
    if candidate_ms <= 0:
        raise ValueError(f"latency must be positive, got {candidate_ms}")
    return baseline_ms / candidate_ms
