"""Row softmax on sm_100a (``kernelforge/kernels/softmax.py:1-157``).

``y_i = exp(x_i - max x) / sum_j exp(x_j - max x)`` with fp32 arithmetic and one
rounding to the input dtype. The row maximum is subtracted for the reason the
reference gives: fp16 ``exp`` overflows above x ~ 11. Both native kernels read
each row once into registers, reduce the (max, sum of exp) pair in a single
pass with the online rescaling rule, and write the row once. Rows of 2 to
32 KB go to the register kernel (one CTA per row, about eight 16-byte vectors
per thread, 0.95-0.99 of the copy bandwidth on B200); with many rows, narrower
and wider rows go to a persistent kernel that streams rows through
shared-memory slots with bulk copies (loads of later rows in flight while
earlier ones reduce); few rows wider than 64 KiB take a cluster of CTAs that
shares the row through distributed shared memory. Unlike the reference's Triton
kernel (capped at 16384 columns) it takes rows up to 131072 columns, which
covers the baseline's 32000-column vocabulary softmax.
"""

from __future__ import annotations

from collections.abc import Callable

import torch

from kernelo_b200.benchmark import metrics
from kernelo_b200.kernels.base import Operator, seeded_generator
from kernelo_b200.kernels.rows_common import MAX_BLOCK_SIZE, check_block, check_row_input, default_rows_config
from kernelo_b200.runtime import native
from kernelo_b200.tuning.config import KernelConfig, Problem
from kernelo_b200.tuning.search import SoftmaxSearchSpace


def default_config(n_cols: int, dtype: torch.dtype = torch.float16, n_rows: int | None = None) -> KernelConfig:
    """The library's choice for contiguous rows (``n_rows`` unknown: the register kernel)."""
    return default_rows_config("softmax", n_cols, dtype, rows=n_rows)


def softmax(x: torch.Tensor, *, config: KernelConfig | None = None) -> torch.Tensor:
    check_row_input(x)
    n_rows, n_cols = x.shape
    if config is None and n_cols <= MAX_BLOCK_SIZE:
        cfg = None  # the library resolves its default itself (default_rows_config mirrors it)
    else:
        cfg = config or default_rows_config("softmax", n_cols, x.dtype, rows=n_rows, x=x,
                                            sm_count=native.sm_count(x.device.index))
        check_block(cfg, n_cols, "row width")
    out = torch.empty((n_rows, n_cols), device=x.device, dtype=x.dtype)
    if n_rows and n_cols:
        native.softmax_rows(x, out, cfg)
    return out


class SoftmaxOperator(Operator):
    name = "softmax"
    config_order = ("ROW_KERNEL", "BLOCK_SIZE", "ROWS_PER_PROGRAM", "num_warps", "CLUSTER", "ROW_GROUPS",
                    "num_stages")

    def __init__(self, *, distribution: str = "baseline") -> None:
        if distribution not in ("baseline", "reference"):
            raise ValueError("distribution must be 'baseline' or 'reference'")
        self.distribution = distribution

    def search_space(self) -> SoftmaxSearchSpace:
        return SoftmaxSearchSpace()

    def make_inputs(self, problem: Problem, device: torch.device, *, seed: int = 0):
        """x ~ N(0, 4^2) (baseline) or N(0, 1) (``distribution="reference"``)."""
        d = problem.dims_dict
        gen = seeded_generator(seed)
        std = 4.0 if self.distribution == "baseline" else 1.0
        x = (torch.randn(d["rows"], d["cols"], generator=gen) * std).to(problem.dtype)
        return (x.to(device),)

    def reference(self, *inputs: torch.Tensor) -> torch.Tensor:
        (x,) = inputs
        return torch.softmax(x, dim=-1)

    def run(self, config: KernelConfig, *inputs: torch.Tensor) -> torch.Tensor:
        (x,) = inputs
        return softmax(x, config=config)

    def default_config(self, problem: Problem) -> KernelConfig:
        return default_config(problem.dims_dict["cols"], problem.dtype, problem.dims_dict["rows"])

    def flops(self, problem: Problem) -> int:
        d = problem.dims_dict
        return 5 * d["rows"] * d["cols"]

    def bytes_moved(self, problem: Problem) -> int:
        d = problem.dims_dict
        return metrics.softmax_bytes(d["rows"], d["cols"], problem.itemsize)

    def is_memory_bound(self) -> bool:
        return True

    def baselines(self, problem: Problem, inputs) -> dict[str, Callable[[], torch.Tensor]]:
        (x,) = inputs
        return {"torch_eager": lambda: torch.softmax(x, dim=-1)}
