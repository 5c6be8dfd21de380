"""Shared host logic of the row kernels (softmax, RMSNorm).

``default_rows_config`` mirrors ``resolve_rows_config`` in ``csrc/rows.cu``:

* a softmax (RMSNorm) over many rows (at least two per SM) of up to 2 KB (4 KB)
  that hold whole 16-byte vectors and start on the 16-byte grid goes to the
  warp-per-row kernel
  (``ROW_KERNEL=3``, ``csrc/rows_warp.cu``): persistent CTAs of 8 warps, a warp
  per row, the next row loaded into registers while the current one is reduced;
* a softmax over many rows whose input and output rows sit at the same
  16-byte phase, with rows of up to 2 KB (not taken by the warp kernel) or
  beyond 32 KB, goes to the persistent streaming kernel (``ROW_KERNEL=2``,
  ``csrc/rows_stream.cu``): row groups of ``num_warps`` warps (the fewest, as a
  power of two, that hold a row at up to 16 vectors a thread) each keeping
  their next rows in flight as bulk copies into shared-memory slots (two slots
  per group for the narrow rows);
* other softmax rows of up to 32 KB go to the register kernel (``ROW_KERNEL=1``,
  ``csrc/rows.cu``) at about eight 16-byte vectors per thread, one CTA per row;
* RMSNorm, and whatever else is left, to the register kernel at about four
  vectors per thread, one CTA per row until a row exceeds 4096 vectors
  (64 KiB), then a power-of-two cluster of CTAs shares it.
"""

from __future__ import annotations

import torch

from kernelo_b200.dtypes import itemsize
from kernelo_b200.tuning.config import KernelConfig
from kernelo_b200.tuning.search import _RowReductionSpace, ceil_div, next_power_of_2

MAX_BLOCK_SIZE = _RowReductionSpace.MAX_BLOCK_SIZE
VECTORS_PER_CTA = 4096

ROW_KERNEL_REGISTER = 1
ROW_KERNEL_STREAM = 2
ROW_KERNEL_WARP = 3
#: Widest rows of the warp-per-row kernel, in 16-byte vectors (mirrors kf_internal.h):
#: the softmax default (2 KB), the RMSNorm default and the kernel's limit (4 KB).
WARP_MAX_VECTORS = 128
WARP_RMSNORM_MAX_VECTORS = 256
#: Warps of one streaming CTA, shared by its row groups.
STREAM_CONSUMER_WARPS = 16
#: Shared memory of one sm_100 CTA, and what the streaming kernel keeps besides its slots.
SM100_SMEM_PER_BLOCK = 232_448
STREAM_FIXED_SMEM = 128 + 8 * 16 * 16 + 16
#: 16-byte vectors a streaming thread may hold.
STREAM_MAX_VECTORS = 16


def stream_default_warps(cols: int, dtype: torch.dtype) -> int:
    nvec = cols * itemsize(dtype) // 16
    warps = min(STREAM_CONSUMER_WARPS, max(1, ceil_div(nvec, 32 * STREAM_MAX_VECTORS)))
    return next_power_of_2(warps)


def stream_vectors_per_thread(cols: int, dtype: torch.dtype, warps: int) -> int:
    return max(1, ceil_div(cols * itemsize(dtype) // 16, 32 * warps))


def stream_fits(cols: int, dtype: torch.dtype) -> bool:
    """Whether one row fits a shared-memory slot and 16 vectors per thread at 16 warps."""
    slot = ceil_div(cols * itemsize(dtype) // 16 * 16, 128) * 128
    if STREAM_FIXED_SMEM + slot + 8 > SM100_SMEM_PER_BLOCK:
        return False
    return stream_vectors_per_thread(cols, dtype, STREAM_CONSUMER_WARPS) <= STREAM_MAX_VECTORS


def same_phase(x: torch.Tensor | None, cols: int) -> bool:
    """x rows at the 16-byte phase of a fresh contiguous output (mirrors rows_stream.cu)."""
    if x is None:
        return True
    size = x.element_size()
    return x.data_ptr() % 16 == 0 and (x.stride(0) * size) % 16 == (cols * size) % 16


def warp_fits(cols: int, dtype: torch.dtype, x: torch.Tensor | None = None, *,
              max_vectors: int = WARP_MAX_VECTORS) -> bool:
    """Rows the warp-per-row kernel takes by default (mirrors rows_warp_supported
    and resolve_rows_config): whole 16-byte vectors, at most ``max_vectors``
    of them, input rows on the 16-byte grid (the output is a fresh contiguous
    tensor, on the grid whenever the rows are whole vectors)."""
    size = itemsize(dtype)
    if (cols * size) % 16 != 0 or cols * size // 16 > max_vectors:
        return False
    return x is None or (x.data_ptr() % 16 == 0 and (x.stride(0) * size) % 16 == 0)


#: Softmax kernel choice by row width in 16-byte vectors (mirrors kf_internal.h).
SOFTMAX_STREAM_MAX_VECTORS = 128
SOFTMAX_REGISTER_MAX_VECTORS = 2048


def default_rows_config(
    operation: str,
    cols: int,
    dtype: torch.dtype,
    *,
    rows: int | None = None,
    x: torch.Tensor | None = None,
    sm_count: int = 148,
) -> KernelConfig:
    """The library's choice (mirrors resolve_rows_config in rows.cu): rows on
    the 16-byte grid go a warp per row up to 2 KB (softmax) or 4 KB (RMSNorm); other
    softmax rows up to 2 KB stream, rows up to 32 KB sit in registers at about
    eight 16-byte vectors per thread, wider rows stream again (when there are
    enough rows for every SM and the kernel takes the layout); RMSNorm uses the
    register kernel at about four vectors per thread."""
    block = next_power_of_2(max(cols, 1))
    nvec = ceil_div(cols * itemsize(dtype), 16)
    warp_max = WARP_RMSNORM_MAX_VECTORS if operation == "rmsnorm" else WARP_MAX_VECTORS
    if rows is not None and rows >= 2 * sm_count and warp_fits(cols, dtype, x, max_vectors=warp_max):
        return KernelConfig(operation, BLOCK_SIZE=block, ROW_KERNEL=ROW_KERNEL_WARP, num_warps=1)
    if operation == "softmax":
        narrow = nvec <= SOFTMAX_STREAM_MAX_VECTORS
        in_registers = nvec <= SOFTMAX_REGISTER_MAX_VECTORS
        if (
            (narrow or not in_registers)
            and rows is not None
            and rows >= 2 * sm_count
            and stream_fits(cols, dtype)
            and same_phase(x, cols)
        ):
            cfg = KernelConfig(
                operation,
                BLOCK_SIZE=block,
                ROW_KERNEL=ROW_KERNEL_STREAM,
                num_warps=stream_default_warps(cols, dtype),
            )
            return cfg.replace(num_stages=2) if narrow else cfg
        if in_registers:
            warps = 1
            while 2 * warps * 256 <= nvec:
                warps *= 2
            while ceil_div(nvec, 32 * warps) > 16:
                warps *= 2
            return KernelConfig(
                operation,
                BLOCK_SIZE=block,
                ROW_KERNEL=ROW_KERNEL_REGISTER,
                ROWS_PER_PROGRAM=1,
                num_warps=warps,
                CLUSTER=1,
            )
    cluster = 1
    if nvec > VECTORS_PER_CTA:
        cluster = next_power_of_2(min(8, ceil_div(nvec, VECTORS_PER_CTA)))
    per_cta = ceil_div(nvec, cluster)
    threads = min(1024, ceil_div(per_cta, 4))
    warps = max(1, min(32, ceil_div(threads, 32)))
    return KernelConfig(
        operation,
        BLOCK_SIZE=block,
        ROW_KERNEL=ROW_KERNEL_REGISTER,
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
