"""Callers of the hot path: a transformer block whose RMSNorms and MLP
up-projection + GELU run on the native kernels
(``kernelforge/integration/__init__.py``)."""

from __future__ import annotations

from kernelo_b200.integration.transformer import (
    BACKEND_KERNELFORGE,
    BACKEND_TORCH,
    BACKENDS,
    BlockConfig,
    TransformerBlock,
    amdahl_breakdown,
    benchmark_block,
)

__all__ = ["BACKENDS", "BACKEND_KERNELFORGE", "BACKEND_TORCH", "BlockConfig", "TransformerBlock",
           "amdahl_breakdown", "benchmark_block"]
