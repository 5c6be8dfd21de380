"""A pre-norm decoder block whose normalisations and MLP activation can run on
the native kernels -- the hot path's first real caller.

The reference measures its kernels inside a transformer block
(``kernelforge/integration/transformer.py:71-187``): the two RMSNorms and the
MLP up-projection with bias + GELU (tanh form) are swapped for the library's
kernels, while attention and the QKV, output and down projections stay
PyTorch, so the comparison isolates the swapped operators. This module keeps
that experiment and its public names (``BlockConfig``, ``TransformerBlock``,
``benchmark_block``, ``amdahl_breakdown``), built its own way:

* the swappable operators live behind two small providers, :class:`_TorchOps`
  and :class:`_NativeOps`, and the block's ``backend`` attribute picks one --
  one module, one set of weights, so a parity check cannot be fooled by
  differing initialisation;
* the native provider resolves a config per (operation, rows, cols) once
  through call-time dispatch (the tuned-config cache, else the library
  default) and reuses it on every later forward;
* :class:`AmdahlBreakdown` states the block speedup the operator speedups
  predict next to the one measured.
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
    """Geometry of one decoder block. The default is Llama-2-7B's matrix shapes
    (4096 hidden, 32 heads, 11008 intermediate) with a bias + GELU MLP, the
    epilogue the fused kernel implements."""

    hidden: int = 4096
    heads: int = 32
    intermediate: int = 11008
    eps: float = DEFAULT_EPS

    def __post_init__(self) -> None:
        if self.hidden % self.heads != 0:
            raise ValueError(f"hidden {self.hidden} is not divisible by {self.heads} heads")

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads


class _TorchOps:
    """The swapped operators as plain PyTorch (the comparison's baseline)."""

    def rms(self, flat: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
        return rmsnorm_reference(flat, weight, eps=eps)

    def up_gelu(self, flat: torch.Tensor, up: nn.Linear) -> torch.Tensor:
        return F.gelu(up(flat), approximate="tanh")


class _NativeOps:
    """The swapped operators on the library's kernels, with one config per
    (operation, rows, cols) resolved through dispatch and then reused."""

    def __init__(self, cache: ConfigCache | None, intermediate: int) -> None:
        self.cache = cache
        self.intermediate = intermediate
        self.selected: dict[tuple[str, int, int], KernelConfig] = {}

    def config(self, operation: str, rows: int, cols: int, dtype: torch.dtype) -> KernelConfig:
        key = (operation, rows, cols)
        found = self.selected.get(key)
        if found is None:
            from kernelo_b200.kernels import get_operator

            dims = dict(rows=rows, cols=cols) if operation == "rmsnorm" else dict(M=rows, N=self.intermediate, K=cols)
            problem = Problem.create(operation, dtype, **dims)
            found = self.selected[key] = select_config(get_operator(operation), problem, cache=self.cache).config
        return found

    def rms(self, flat: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
        return rmsnorm(flat, weight, eps=eps, config=self.config("rmsnorm", *flat.shape, flat.dtype))

    def up_gelu(self, flat: torch.Tensor, up: nn.Linear) -> torch.Tensor:
        # nn.Linear keeps W as [N, K]: its transposed view is a K-major B, read without a copy
        return fused_linear_gelu(flat, up.weight.t(), up.bias,
                                 config=self.config("fused_linear", *flat.shape, flat.dtype))


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
        self.config = config if config is not None else BlockConfig()
        self._providers = {BACKEND_TORCH: _TorchOps(), BACKEND_KERNELFORGE: _NativeOps(cache, self.config.intermediate)}
        self.backend = backend
        h, i = self.config.hidden, self.config.intermediate
        like = {"device": device, "dtype": dtype}
        self.attn_norm_weight = nn.Parameter(torch.ones(h, **like))
        self.mlp_norm_weight = nn.Parameter(torch.ones(h, **like))
        self.qkv_proj = nn.Linear(h, 3 * h, bias=False, **like)
        self.out_proj = nn.Linear(h, h, bias=False, **like)
        self.mlp_up = nn.Linear(h, i, bias=True, **like)
        self.mlp_down = nn.Linear(i, h, bias=False, **like)

    @property
    def backend(self) -> str:
        return self._backend

    @backend.setter
    def backend(self, name: str) -> None:
        if name not in BACKENDS:
            raise ValueError(f"backend must be one of {BACKENDS}, got {name!r}")
        self._backend = name

    @property
    def ops(self) -> _TorchOps | _NativeOps:
        return self._providers[self._backend]

    @property
    def resolved_configs(self) -> dict[tuple[str, int, int], KernelConfig]:
        """The native configs resolved so far, by (operation, rows, cols)."""
        return dict(self._providers[BACKEND_KERNELFORGE].selected)

    def norm(self, flat: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
        """RMSNorm of [tokens, hidden] under the current backend."""
        return self.ops.rms(flat, weight, self.config.eps)

    def mlp_activation(self, flat: torch.Tensor) -> torch.Tensor:
        """gelu_tanh(flat @ W_up^T + b_up) under the current backend."""
        return self.ops.up_gelu(flat, self.mlp_up)

    def _attention(self, normed: torch.Tensor) -> torch.Tensor:
        """Causal multi-head self-attention of [batch, seq, hidden] (always PyTorch)."""
        b, s, h = normed.shape
        heads = self.config.heads
        q, k, v = self.qkv_proj(normed).view(b, s, 3, heads, h // heads).permute(2, 0, 3, 1, 4).unbind(0)
        mixed = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        return self.out_proj(mixed.transpose(1, 2).reshape(b, s, h))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.ndim != 3:
            raise ValueError(f"expected (batch, seq, hidden), got {tuple(x.shape)}")
        b, s, h = x.shape
        if h != self.config.hidden:
            raise ValueError(f"expected hidden {self.config.hidden}, got {h}")
        tokens = b * s
        x = x + self._attention(self.norm(x.reshape(tokens, h), self.attn_norm_weight).view(b, s, h))
        mlp_in = self.norm(x.reshape(tokens, h), self.mlp_norm_weight)
        return x + self.mlp_down(self.mlp_activation(mlp_in)).view(b, s, h)


def _timed(call, *, device, warmup: int, iterations: int):
    from kernelo_b200.benchmark.runner import benchmark

    # no L2 flush: a block's working set is far larger than the L2
    return benchmark(call, warmup=warmup, iterations=iterations, device=device, flush_l2=False)


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
    """One block timed under each backend, on the same weights and input."""
    block = TransformerBlock(config, dtype=dtype, device=device, cache=cache)
    x = torch.randn(batch, seq, block.config.hidden, device=device, dtype=dtype)
    timings: dict[str, object] = {}
    with torch.inference_mode():
        for name in BACKENDS:
            block.backend = name
            timings[name] = _timed(lambda: block(x), device=device, warmup=warmup, iterations=iterations)
    return timings


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
        """Amdahl's law: the untouched share keeps its time, the swapped share
        shrinks by the operator speedup."""
        share = self.swapped_share
        return 1.0 / ((1.0 - share) + share / self.operator_speedup)

    @property
    def measured_block_speedup(self) -> float:
        return self.block_ms[BACKEND_TORCH] / self.block_ms[BACKEND_KERNELFORGE]

    def render(self) -> str:
        t, n = BACKEND_TORCH, BACKEND_KERNELFORGE
        return (f"block            torch {self.block_ms[t]:.3f} ms   kernelforge {self.block_ms[n]:.3f} ms\n"
                f"swapped ops      torch {self.swapped_ms[t]:.3f} ms   kernelforge {self.swapped_ms[n]:.3f} ms   "
                f"({self.operator_speedup:.2f}x)\n"
                f"swapped share of the torch block: {100 * self.swapped_share:.1f} %\n"
                f"block speedup: predicted {self.predicted_block_speedup:.3f}x (Amdahl), "
                f"measured {self.measured_block_speedup:.3f}x")


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
    """The whole block and its swapped operators alone (both RMSNorms and the
    MLP up-projection + GELU, on the block's own weights and shapes), timed
    under each backend."""
    block = TransformerBlock(config, dtype=dtype, device=device, cache=cache)
    h = block.config.hidden
    x = torch.randn(batch, seq, h, device=device, dtype=dtype)
    flat = torch.randn(batch * seq, h, device=device, dtype=dtype)

    def swapped_only() -> torch.Tensor:
        block.norm(flat, block.attn_norm_weight)
        return block.mlp_activation(block.norm(flat, block.mlp_norm_weight))

    whole: dict[str, float] = {}
    parts: dict[str, float] = {}
    with torch.inference_mode():
        for name in BACKENDS:
            block.backend = name
            whole[name] = _timed(lambda: block(x), device=device, warmup=warmup, iterations=iterations).median_ms
            parts[name] = _timed(swapped_only, device=device, warmup=warmup, iterations=iterations).median_ms
    return AmdahlBreakdown(whole, parts)
