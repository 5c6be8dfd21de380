"""Shared host logic of the row kernels (softmax, RMSNorm).

``default_rows_config`` mirrors ``resolve_rows_config`` in ``csrc/rows.cu``:
about four 16-byte vectors per thread, one CTA per row until a row exceeds
4096 vectors (64 KiB), then a power-of-two cluster of CTAs shares it.
"""

from __future__ import annotations

import torch

from kernelo_b200.dtypes import itemsize
from kernelo_b200.tuning.config import KernelConfig
from kernelo_b200.tuning.search import _RowReductionSpace, ceil_div, next_power_of_2

MAX_BLOCK_SIZE = _RowReductionSpace.MAX_BLOCK_SIZE
VECTORS_PER_CTA = 4096


def default_rows_config(operation: str, cols: int, dtype: torch.dtype) -> KernelConfig:
    nvec = ceil_div(cols * itemsize(dtype), 16)
    cluster = 1
    if nvec > VECTORS_PER_CTA:
        cluster = next_power_of_2(min(8, ceil_div(nvec, VECTORS_PER_CTA)))
    per_cta = ceil_div(nvec, cluster)
    threads = min(1024, ceil_div(per_cta, 4))
    warps = max(1, min(32, ceil_div(threads, 32)))
    return KernelConfig(
        operation,
        BLOCK_SIZE=next_power_of_2(max(cols, 1)),
        ROWS_PER_PROGRAM=1,
        num_warps=warps,
        CLUSTER=cluster,
    )


def check_row_input(x: torch.Tensor) -> None:
    if x.ndim != 2:
        raise ValueError(f"expected a 2D tensor, got shape {tuple(x.shape)}")
    if x.shape[1] > 1 and x.stride(1) != 1:
        raise ValueError(
            "x must have a contiguous last dimension; the kernel indexes columns "
            "directly off the row pointer. Pass x.contiguous() -- explicitly, so the "
            "copy is not hidden inside a measured region."
        )
    if x.device.type != "cuda":
        raise ValueError(f"x must be a CUDA tensor, got {x.device}")


def check_block(config: KernelConfig, cols: int, what: str) -> None:
    block = config.get("BLOCK_SIZE", next_power_of_2(max(cols, 1)))
    if block < cols:
        raise ValueError(
            f"BLOCK_SIZE={block} cannot hold a row of {cols}; this kernel is single-pass by design"
        )
    if block > MAX_BLOCK_SIZE:
        raise ValueError(f"{what} {cols} exceeds the single-pass limit of {MAX_BLOCK_SIZE}")
