"""Blocked GEMM ``C = A @ B`` on sm_100a (``kernelforge/kernels/matmul.py:54-259``).

Same contract as the reference wrapper -- 2-D operands of one dtype, strides
honoured (transposed views need no copy), output allocated here in the input
dtype, fp32 accumulation, fp32 operands computed in IEEE fp32 -- executed by
the native library: the persistent TMA + tcgen05 kernel for fp16/bf16 operands
a TMA tensor map can describe, the CUDA-core kernel otherwise (fp32, odd K or N
such as 4099 or 509, unaligned views).
"""

from __future__ import annotations

from collections.abc import Callable

import torch

from kernelo_b200.benchmark import metrics
from kernelo_b200.kernels import gemm_common as gc
from kernelo_b200.kernels.base import Operator, seeded_generator
from kernelo_b200.runtime import native
from kernelo_b200.testing import exact_fp32_matmul
from kernelo_b200.tuning.config import KernelConfig, Problem
from kernelo_b200.tuning.search import MatmulSearchSpace


def _check_operands(a: torch.Tensor, b: torch.Tensor) -> None:
    if a.ndim != 2 or b.ndim != 2:
        raise ValueError(f"expected 2D operands, got {tuple(a.shape)} and {tuple(b.shape)}")
    if a.shape[1] != b.shape[0]:
        raise ValueError(f"shape mismatch for matmul: {tuple(a.shape)} @ {tuple(b.shape)}")
    if a.dtype != b.dtype:
        raise ValueError(f"dtype mismatch: {a.dtype} vs {b.dtype}")
    if a.device != b.device or a.device.type != "cuda":
        raise ValueError(f"operands must be CUDA tensors on one device, got {a.device} and {b.device}")


def matmul(a: torch.Tensor, b: torch.Tensor, *, config: KernelConfig | None = None) -> torch.Tensor:
    """``a @ b`` through the native library; ``config=None`` lets it choose."""
    _check_operands(a, b)
    m, _ = a.shape
    n = b.shape[1]
    c = torch.empty((m, n), device=a.device, dtype=a.dtype)
    if m and n:
        native.gemm(a, b, c, launch=native.GemmLaunch.from_config(config))
    return c


def default_config(m: int, n: int, k: int, dtype: torch.dtype, *, sm_count: int = 148) -> KernelConfig:
    """The config the library picks for contiguous row-major A [M,K] and B [K,N]."""
    return gc.default_gemm_config("matmul", m, n, k, dtype, b_layout="kn", sm_count=sm_count)


class MatmulOperator(Operator):
    name = "matmul"
    config_order = ("KERNEL", "BLOCK_M", "BLOCK_N", "BLOCK_K", "GROUP_M", "num_stages", "STREAM_K",
                    "SWAP_AB", "CLUSTER_M", "CLUSTER_N")

    def search_space(self) -> MatmulSearchSpace:
        return MatmulSearchSpace()

    def make_inputs(self, problem: Problem, device: torch.device, *, seed: int = 0):
        d = problem.dims_dict
        gen = seeded_generator(seed)
        a = torch.randn(d["M"], d["K"], generator=gen).to(problem.dtype)
        b = torch.randn(d["K"], d["N"], generator=gen).to(problem.dtype)
        return a.to(device), b.to(device)

    def reference(self, *inputs: torch.Tensor) -> torch.Tensor:
        a, b = inputs
        with exact_fp32_matmul():
            return torch.matmul(a, b)

    def run(self, config: KernelConfig, *inputs: torch.Tensor) -> torch.Tensor:
        a, b = inputs
        return matmul(a, b, config=config)

    def default_config(self, problem: Problem) -> KernelConfig:
        d = problem.dims_dict
        return default_config(d["M"], d["N"], d["K"], problem.dtype)

    def flops(self, problem: Problem) -> int:
        d = problem.dims_dict
        return metrics.matmul_flops(d["M"], d["N"], d["K"])

    def bytes_moved(self, problem: Problem) -> int:
        d = problem.dims_dict
        return metrics.matmul_bytes(d["M"], d["N"], d["K"], problem.itemsize)

    def baselines(self, problem: Problem, inputs) -> dict[str, Callable[[], torch.Tensor]]:
        a, b = inputs
        default = self.default_config(problem)
        return {
            "torch_eager": lambda: torch.matmul(a, b),
            "kernelforge_default": lambda: matmul(a, b, config=default),
        }
