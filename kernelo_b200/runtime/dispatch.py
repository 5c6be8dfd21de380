"""Config selection at call time (``kernelforge/runtime/dispatch.py:47-64``).

A cache read, never a tuning run: a hit returns the tuned config for this
device, a miss the operator's default, and the source is reported either way.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from kernelo_b200.kernels.base import Operator
from kernelo_b200.runtime.env import device_key as resolve_device_key
from kernelo_b200.tuning.cache import ConfigCache
from kernelo_b200.tuning.config import KernelConfig, Problem

SOURCE_CACHE = "cache"
SOURCE_DEFAULT = "default"


@dataclass(frozen=True)
class Selection:
    config: KernelConfig
    source: str
    device_key: str

    @property
    def tuned(self) -> bool:
        return self.source == SOURCE_CACHE

    def describe(self) -> str:
        if self.tuned:
            return f"tuned configuration for {self.device_key}"
        return f"default configuration (no cache entry for {self.device_key})"


def select_config(
    operator: Operator,
    problem: Problem,
    *,
    cache: ConfigCache | None = None,
    device: torch.device | str | None = None,
) -> Selection:
    key = resolve_device_key(device)
    store = cache if cache is not None else ConfigCache()
    hit = store.get(problem, key)
    if hit is not None:
        return Selection(hit, SOURCE_CACHE, key)
    return Selection(operator.default_config(problem), SOURCE_DEFAULT, key)
