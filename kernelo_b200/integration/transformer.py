"""A pre-norm decoder block whose normalisations and MLP activation run on the
native kernels (``kernelforge/integration/transformer.py:1-187``).

The block is the first real caller of the hot path: dispatch picks a config
per shape (cache, else the library default), then RMSNorm and the fused
linear + bias + GELU run as B200 kernels. What is swapped, as in the
reference:

* both RMSNorms, and the MLP up-projection with its bias and GELU (tanh form)
  folded into the GEMM epilogue;
* not attention (``scaled_dot_product_attention``) and not the QKV, output
  and down projections (``nn.Linear``), so the comparison isolates the
  swapped operators.

Both backends share one module and one set of weights: ``backend`` is a
mutable attribute, so a parity check cannot be fooled by differing
initialisation. :func:`amdahl_breakdown` times the swapped operators alone
and the whole block under each backend, and states the block speedup the
operator speedups predict next to the one measured.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn

from kernelo_b200.kernels.fused_linear import fused_linear_gelu
from kernelo_b200.kernels.rmsnorm import DEFAULT_EPS, rmsnorm, rmsnorm_reference
from kernelo_b200.runtime.dispatch import select_config
from kernelo_b200.tuning.cache import ConfigCache
from kernelo_b200.tuning.config import KernelConfig, Problem

BACKEND_TORCH = "torch"
BACKEND_KERNELFORGE = "kernelforge"
BACKENDS = (BACKEND_TORCH, BACKEND_KERNELFORGE)


@dataclass(frozen=True)
class BlockConfig:
    """Geometry of one decoder block; the default is Llama-2-7B's (4096 hidden,
    32 heads, 11008 intermediate) with a GELU MLP, since the fused epilogue is
    bias + GELU -- the matrix shapes are the real ones."""

    hidden: int = 4096
    heads: int = 32
    intermediate: int = 11008
    eps: float = DEFAULT_EPS

    def __post_init__(self) -> None:
        if self.hidden % self.heads:
            raise ValueError(f"hidden {self.hidden} is not divisible by {self.heads} heads")

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads


class TransformerBlock(nn.Module):
    """Pre-norm decoder block with swappable normalisation and MLP activation."""

    def __init__(
        self,
        config: BlockConfig | None = None,
        *,
        dtype: torch.dtype = torch.float16,
        device: torch.device | str = "cuda",
        backend: str = BACKEND_TORCH,
        cache: ConfigCache | None = None,
    ) -> None:
        super().__init__()
        if backend not in BACKENDS:
            raise ValueError(f"backend must be one of {BACKENDS}, got {backend!r}")
        self.config = config or BlockConfig()
        self.backend = backend
        self._cache = cache
        # Config lookups read the cache file: resolved once per shape, not per forward.
        self._selected: dict[tuple[str, int, int], KernelConfig] = {}
        hidden, intermediate = self.config.hidden, self.config.intermediate
        factory = {"device": device, "dtype": dtype}
        self.attn_norm_weight = nn.Parameter(torch.ones(hidden, **factory))
        self.mlp_norm_weight = nn.Parameter(torch.ones(hidden, **factory))
        self.qkv_proj = nn.Linear(hidden, 3 * hidden, bias=False, **factory)
        self.out_proj = nn.Linear(hidden, hidden, bias=False, **factory)
        self.mlp_up = nn.Linear(hidden, intermediate, bias=True, **factory)
        self.mlp_down = nn.Linear(intermediate, hidden, bias=False, **factory)

    def _config_for(self, operation: str, rows: int, cols: int, dtype: torch.dtype) -> KernelConfig:
        key = (operation, rows, cols)
        if key not in self._selected:
            from kernelo_b200.kernels import get_operator

            if operation == "rmsnorm":
                problem = Problem.create(operation, dtype, rows=rows, cols=cols)
            else:
                problem = Problem.create(operation, dtype, M=rows, N=self.config.intermediate, K=cols)
            self._selected[key] = select_config(get_operator(operation), problem, cache=self._cache).config
        return self._selected[key]

    def norm(self, flat: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
        """RMSNorm of [tokens, hidden] under the current backend."""
        if self.backend == BACKEND_TORCH:
            return rmsnorm_reference(flat, weight, eps=self.config.eps)
        config = self._config_for("rmsnorm", flat.shape[0], flat.shape[1], flat.dtype)
        return rmsnorm(flat, weight, eps=self.config.eps, config=config)

    def mlp_activation(self, flat: torch.Tensor) -> torch.Tensor:
        """gelu_tanh(flat @ W_up^T + b_up) under the current backend."""
        if self.backend == BACKEND_TORCH:
            return F.gelu(self.mlp_up(flat), approximate="tanh")
        config = self._config_for("fused_linear", flat.shape[0], flat.shape[1], flat.dtype)
        # nn.Linear stores [N, K]; its transposed view is the kernel's K-major B, no copy.
        return fused_linear_gelu(flat, self.mlp_up.weight.t(), self.mlp_up.bias, config=config)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.ndim != 3:
            raise ValueError(f"expected (batch, seq, hidden), got {tuple(x.shape)}")
        batch, seq, hidden = x.shape
        if hidden != self.config.hidden:
            raise ValueError(f"expected hidden {self.config.hidden}, got {hidden}")
        heads, head_dim = self.config.heads, self.config.head_dim
        normed = self.norm(x.reshape(batch * seq, hidden), self.attn_norm_weight)
        qkv = self.qkv_proj(normed.view(batch, seq, hidden))
        q, k, v = (t.view(batch, seq, heads, head_dim).transpose(1, 2) for t in qkv.split(hidden, dim=-1))
        attended = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        x = x + self.out_proj(attended.transpose(1, 2).reshape(batch, seq, hidden))
        normed = self.norm(x.reshape(batch * seq, hidden), self.mlp_norm_weight)
        return x + self.mlp_down(self.mlp_activation(normed)).view(batch, seq, hidden)


def benchmark_block(
    config: BlockConfig | None = None,
    *,
    batch: int = 1,
    seq: int = 2048,
    dtype: torch.dtype = torch.float16,
    device: torch.device | str = "cuda",
    warmup: int = 25,
    iterations: int = 100,
    cache: ConfigCache | None = None,
) -> dict[str, object]:
    """Time one block per backend on identical weights and inputs (no L2
    flush: the block's working set is far larger than the L2)."""
    from kernelo_b200.benchmark.runner import benchmark

    block = TransformerBlock(config, dtype=dtype, device=device, cache=cache)
    x = torch.randn(batch, seq, block.config.hidden, device=device, dtype=dtype)
    results: dict[str, object] = {}
    with torch.inference_mode():
        for backend in BACKENDS:
            block.backend = backend
            results[backend] = benchmark(lambda: block(x), warmup=warmup, iterations=iterations,
                                         device=device, flush_l2=False)
    return results


@dataclass(frozen=True)
class AmdahlBreakdown:
    """Median ms per backend for the block and for its swapped operators."""

    block_ms: dict[str, float]
    swapped_ms: dict[str, float]  # 2 x RMSNorm + MLP up-projection with GELU

    @property
    def swapped_share(self) -> float:
        """Share of the torch block's time the swapped operators held."""
        return self.swapped_ms[BACKEND_TORCH] / self.block_ms[BACKEND_TORCH]

    @property
    def operator_speedup(self) -> float:
        return self.swapped_ms[BACKEND_TORCH] / self.swapped_ms[BACKEND_KERNELFORGE]

    @property
    def predicted_block_speedup(self) -> float:
        """Amdahl: the untouched remainder plus the swapped operators' new time."""
        torch_ms = self.block_ms[BACKEND_TORCH]
        rest = torch_ms - self.swapped_ms[BACKEND_TORCH]
        return torch_ms / (rest + self.swapped_ms[BACKEND_KERNELFORGE])

    @property
    def measured_block_speedup(self) -> float:
        return self.block_ms[BACKEND_TORCH] / self.block_ms[BACKEND_KERNELFORGE]

    def render(self) -> str:
        return "\n".join([
            f"block            torch {self.block_ms[BACKEND_TORCH]:.3f} ms   "
            f"kernelforge {self.block_ms[BACKEND_KERNELFORGE]:.3f} ms",
            f"swapped ops      torch {self.swapped_ms[BACKEND_TORCH]:.3f} ms   "
            f"kernelforge {self.swapped_ms[BACKEND_KERNELFORGE]:.3f} ms   "
            f"({self.operator_speedup:.2f}x)",
            f"swapped share of the torch block: {100 * self.swapped_share:.1f} %",
            f"block speedup: predicted {self.predicted_block_speedup:.3f}x (Amdahl), "
            f"measured {self.measured_block_speedup:.3f}x",
        ])


def amdahl_breakdown(
    config: BlockConfig | None = None,
    *,
    batch: int = 1,
    seq: int = 2048,
    dtype: torch.dtype = torch.float16,
    device: torch.device | str = "cuda",
    warmup: int = 10,
    iterations: int = 50,
    cache: ConfigCache | None = None,
) -> AmdahlBreakdown:
    """Time the whole block and its swapped operators alone (both RMSNorms and
    the MLP up-projection + GELU, on the block's own weights and shapes),
    under each backend."""
    from kernelo_b200.benchmark.runner import benchmark

    block = TransformerBlock(config, dtype=dtype, device=device, cache=cache)
    hidden = block.config.hidden
    x = torch.randn(batch, seq, hidden, device=device, dtype=dtype)
    flat = torch.randn(batch * seq, hidden, device=device, dtype=dtype)

    def swapped() -> torch.Tensor:
        block.norm(flat, block.attn_norm_weight)
        normed = block.norm(flat, block.mlp_norm_weight)
        return block.mlp_activation(normed)

    block_ms: dict[str, float] = {}
    swapped_ms: dict[str, float] = {}
    with torch.inference_mode():
        for backend in BACKENDS:
            block.backend = backend
            block_ms[backend] = benchmark(lambda: block(x), warmup=warmup, iterations=iterations,
                                          device=device, flush_l2=False).median_ms
            swapped_ms[backend] = benchmark(swapped, warmup=warmup, iterations=iterations,
                                            device=device, flush_l2=False).median_ms
    return AmdahlBreakdown(block_ms, swapped_ms)
