"""The operator contract (``kernelforge/kernels/base.py:21-94``).

The tuner is generic: it asks an operator for its search space, reproducible
inputs, a reference result and a way to run one configuration. ``run`` here
reaches the sm_100a kernels through the C ABI instead of a Triton launch;
``reference`` stays the PyTorch computation the reference gates against.
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from collections.abc import Callable

import torch

from kernelo_b200.tuning.config import KernelConfig, Problem
from kernelo_b200.tuning.search import SearchSpace


class Operator(ABC):
    """One tunable operation."""

    name: str
    #: Preferred key order when rendering a config.
    config_order: tuple[str, ...] = ()

    @abstractmethod
    def search_space(self) -> SearchSpace: ...

    @abstractmethod
    def make_inputs(
        self, problem: Problem, device: torch.device, *, seed: int = 0
    ) -> tuple[torch.Tensor, ...]:
        """Reproducible inputs for ``problem`` on ``device``."""

    @abstractmethod
    def reference(self, *inputs: torch.Tensor) -> torch.Tensor:
        """The PyTorch computation this kernel must agree with."""

    @abstractmethod
    def run(self, config: KernelConfig, *inputs: torch.Tensor) -> torch.Tensor:
        """Run the native kernel with ``config``."""

    @abstractmethod
    def default_config(self, problem: Problem) -> KernelConfig:
        """An always-feasible configuration: the untuned baseline and the cache-miss fallback."""

    @abstractmethod
    def flops(self, problem: Problem) -> int: ...

    @abstractmethod
    def bytes_moved(self, problem: Problem) -> int:
        """Minimum global-memory traffic of a perfect kernel, in bytes."""

    def baselines(
        self, problem: Problem, inputs: tuple[torch.Tensor, ...]
    ) -> dict[str, Callable[[], torch.Tensor]]:
        """Comparison implementations by label; ``torch_eager`` is always present."""
        return {"torch_eager": lambda: self.reference(*inputs)}

    def is_memory_bound(self) -> bool:
        return False


def compiled_baseline(
    fn: Callable[..., torch.Tensor], inputs: tuple[torch.Tensor, ...], *, mode: str | None = None
) -> Callable[[], torch.Tensor]:
    """``torch.compile(fn)`` warmed up once, as a comparison label (not a hot path)."""
    compiled = torch.compile(fn, mode=mode) if mode else torch.compile(fn)

    def run() -> torch.Tensor:
        return compiled(*inputs)

    run()
    return run


def seeded_generator(seed: int) -> torch.Generator:
    """A CPU generator: inputs are drawn on the host so they are identical on every machine."""
    return torch.Generator(device="cpu").manual_seed(seed)
