"""Decode-shape GEMM ``Y[M,N] = X[M,K] @ W^T`` for M in 1..256.

The reference has no dedicated kernel: single-token decoding calls its blocked
GEMM with M=1 (``kernelforge/kernels/matmul.py:132`` with BLOCK_M=16, one tile
row), and README.md:666-670 lists split-K as future work. This shape moves
90 MB of weight for 90 MFLOP (1 FLOP/byte), so it is bound by HBM, not by the
tensor cores. Three sm_100a kernels, chosen by the library:

* fp16/bf16 x with up to 32 rows and a K-contiguous [N,K] weight (K % 8 == 0):
  the 16-row tile kernel (``KERNEL=4``, ``csrc/gemv_mma.cu``). One CTA per 16
  weight rows, K split over its warps; lanes stream the rows with contiguous
  loads straight into ``mma.sync`` fragments (0.84 / 0.80 / 0.76 of the copy
  bandwidth at M = 1 / 4 / 16 on B200; at M = 32 24 us against 27 us for the
  tcgen05 GEMV).
* fp32 x with M <= 2: the warp-per-row CUDA-core kernel (``KERNEL=3``,
  ``csrc/gemv_rows.cu``), packed fp32x2 FMAs against x held in shared memory;
  it takes M <= 4 when asked for.
* otherwise (a [K,N] weight, unaligned rows, M > 32): the tcgen05 GEMM with A
  and B swapped -- the weight becomes the 128-row MMA operand -- and K split
  evenly over every SM (stream-K); the last CTA to finish a tile sums the
  partials in a fixed order.

W may be stored [N,K] (``w_layout="nk"``, nn.Linear, the baseline layout) or
[K,N] (``"kn"``, the reference's ``matmul(x, w)`` orientation).
"""

from __future__ import annotations

import dataclasses
from collections.abc import Callable

import torch

from kernelo_b200.benchmark import metrics
from kernelo_b200.dtypes import itemsize
from kernelo_b200.kernels import gemm_common as gc
from kernelo_b200.kernels.base import Operator, seeded_generator
from kernelo_b200.runtime import native
from kernelo_b200.testing import exact_fp32_matmul
from kernelo_b200.tuning.config import KernelConfig, Problem
from kernelo_b200.tuning.search import GemvSearchSpace

MAX_ROWS = 256


def gemv(
    x: torch.Tensor,
    w: torch.Tensor,
    *,
    w_layout: str = "nk",
    config: KernelConfig | None = None,
    out: torch.Tensor | None = None,
    overlap: bool = False,
) -> torch.Tensor:
    """``x @ w.T`` (``"nk"``) or ``x @ w`` (``"kn"``) for a handful of rows.

    ``overlap=True`` promises that ``w`` is not written by the kernel queued
    just before this call on the stream (a model weight): the decode kernels
    then launch as that kernel's CTAs finish and stream the weight while it
    completes, and wait for it before reading ``x`` or writing ``out``
    (programmatic dependent launch; back-to-back GEMVs overlap their tails).
    """
    if x.ndim != 2 or w.ndim != 2:
        raise ValueError(f"expected 2D x and w, got {tuple(x.shape)} and {tuple(w.shape)}")
    if w_layout not in ("nk", "kn"):
        raise ValueError(f"w_layout must be 'nk' or 'kn', got {w_layout!r}")
    k = x.shape[1]
    k_w = w.shape[1] if w_layout == "nk" else w.shape[0]
    n = w.shape[0] if w_layout == "nk" else w.shape[1]
    if k != k_w:
        raise ValueError(f"shape mismatch: x {tuple(x.shape)} against w {tuple(w.shape)} ({w_layout})")
    if x.dtype != w.dtype:
        raise ValueError(f"dtype mismatch: {x.dtype} vs {w.dtype}")
    if x.device != w.device or x.device.type != "cuda":
        raise ValueError("x and w must be CUDA tensors on one device")
    m = x.shape[0]
    if m > MAX_ROWS:
        raise ValueError(f"gemv takes at most {MAX_ROWS} rows, got {m}; use matmul")
    if out is None:
        out = torch.empty((m, n), device=x.device, dtype=x.dtype)
    if m and n:
        launch = native.GemmLaunch.from_config(config)
        if overlap:
            launch = dataclasses.replace(launch, overlap=1)
        native.gemv(x, w, out, w_layout=w_layout, launch=launch)
    return out


def default_config(m: int, n: int, k: int, dtype: torch.dtype, *, sm_count: int = 148) -> KernelConfig:
    """The library's choice for contiguous [M,K] x and [N,K] w (mirrors kf_gemv)."""
    if gc.tile_stream_reject(m, k, dtype) is None and gc.tile_stream_preferred(m, n, k, sm_count=sm_count):
        return KernelConfig("gemv", KERNEL=gc.KERNEL_TILE_STREAM, BLOCK_K=gc.TILE_STREAM_CHUNKS[0])
    if gc.tile_rows_reject(m, k, dtype) is None:
        warps, pairs = gc.tile_rows_default(m)
        return KernelConfig("gemv", KERNEL=gc.KERNEL_TILE_ROWS, BLOCK_M=warps, num_stages=pairs)
    if 1 <= m <= gc.WARP_ROWS_AUTO_MAX_M and gc.warp_rows_smem_bytes(m, k, itemsize(dtype)) <= gc.SM100_SMEM_PER_BLOCK:
        return KernelConfig("gemv", KERNEL=gc.KERNEL_WARP_ROWS)
    aligned = dtype in (torch.float16, torch.bfloat16) and gc.tma_misfit(m, n, k, b_layout="nk") is None
    if not aligned and not gc.packs_by_default(m, n, k, dtype, b_layout="nk"):
        return gc.default_simt_config("gemv", m, n, sm_count=sm_count)
    cfg = gc.default_tcgen05_config("gemv", m, n, max(k, 8), b_layout="nk", sm_count=sm_count)
    # Always swap and split K: the weight streams through every SM.
    return cfg.replace(SWAP_AB=1, STREAM_K=1)


class GemvOperator(Operator):
    name = "gemv"
    config_order = ("KERNEL", "BLOCK_M", "BLOCK_N", "BLOCK_K", "num_stages", "STREAM_K", "SWAP_AB")

    def search_space(self) -> GemvSearchSpace:
        return GemvSearchSpace()

    def make_inputs(self, problem: Problem, device: torch.device, *, seed: int = 0):
        """X ~ N(0,1) [M,K]; W ~ N(0,1/K) stored [N,K]."""
        d = problem.dims_dict
        gen = seeded_generator(seed)
        x = torch.randn(d["M"], d["K"], generator=gen).to(problem.dtype)
        w = (torch.randn(d["N"], d["K"], generator=gen) * d["K"] ** -0.5).to(problem.dtype)
        return x.to(device), w.to(device)

    def reference(self, *inputs: torch.Tensor) -> torch.Tensor:
        x, w = inputs
        with exact_fp32_matmul():
            return torch.matmul(x, w.t())

    def run(self, config: KernelConfig, *inputs: torch.Tensor) -> torch.Tensor:
        x, w = inputs
        return gemv(x, w, config=config)

    def default_config(self, problem: Problem) -> KernelConfig:
        d = problem.dims_dict
        return default_config(d["M"], d["N"], d["K"], problem.dtype)

    def flops(self, problem: Problem) -> int:
        d = problem.dims_dict
        return metrics.matmul_flops(d["M"], d["N"], d["K"])

    def bytes_moved(self, problem: Problem) -> int:
        d = problem.dims_dict
        return metrics.gemv_bytes(d["M"], d["N"], d["K"], problem.itemsize)

    def is_memory_bound(self) -> bool:
        return True

    def baselines(self, problem: Problem, inputs) -> dict[str, Callable[[], torch.Tensor]]:
        x, w = inputs
        return {"torch_eager": lambda: torch.matmul(x, w.t())}
