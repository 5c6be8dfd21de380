"""Which config a call runs with: a cache lookup, never a tuning run.

Keeps the reference's call-time contract (``kernelforge/runtime/dispatch.py:47-64``):
``select_config(operator, problem)`` answers from the tuned-config cache when
this device has an entry for the problem, and with the operator's default
otherwise, and says which of the two it was.

Serving calls this on every forward pass, so the lookup is kept off the file
system: without an explicit cache the default cache file is parsed once per
process and parsed again only when the file on disk changes (its size or
modification time), and the device key is resolved once per device.
"""

from __future__ import annotations

import os
from dataclasses import dataclass

import torch

from kernelo_b200.kernels.base import Operator
from kernelo_b200.runtime.env import device_key as resolve_device_key
from kernelo_b200.tuning.cache import ConfigCache, default_cache_path
from kernelo_b200.tuning.config import KernelConfig, Problem

SOURCE_CACHE = "cache"
SOURCE_DEFAULT = "default"


@dataclass(frozen=True)
class Selection:
    """The config to run, where it came from, and the device it was looked up for."""

    config: KernelConfig
    source: str
    device_key: str

    @property
    def tuned(self) -> bool:
        return self.source == SOURCE_CACHE

    def describe(self) -> str:
        if not self.tuned:
            return f"default configuration (no cache entry for {self.device_key})"
        return f"tuned configuration for {self.device_key}"


class _DefaultCache:
    """The default cache file, parsed again only when it changes on disk."""

    def __init__(self) -> None:
        self._stamp: tuple | None = None
        self._cache: ConfigCache | None = None

    def get(self) -> ConfigCache:
        path = default_cache_path()
        try:
            st = os.stat(path)
            stamp = (str(path), st.st_size, st.st_mtime_ns)
        except FileNotFoundError:
            stamp = (str(path), None, None)
        if self._cache is None or stamp != self._stamp:
            self._cache, self._stamp = ConfigCache(path), stamp
        return self._cache


_DEFAULT_CACHE = _DefaultCache()
_DEVICE_KEYS: dict[str, str] = {}


def _device_key(device: torch.device | str | None) -> str:
    if device is None and torch.cuda.is_available():
        device = torch.device("cuda", torch.cuda.current_device())
    tag = str(device)
    key = _DEVICE_KEYS.get(tag)
    if key is None:
        key = _DEVICE_KEYS[tag] = resolve_device_key(device)
    return key


def select_config(
    operator: Operator,
    problem: Problem,
    *,
    cache: ConfigCache | None = None,
    device: torch.device | str | None = None,
) -> Selection:
    """The tuned config of ``problem`` on ``device`` if the cache has one, else the default."""
    key = _device_key(device)
    store = cache if cache is not None else _DEFAULT_CACHE.get()
    tuned = store.get(problem, key)
    if tuned is None:
        return Selection(operator.default_config(problem), SOURCE_DEFAULT, key)
    return Selection(tuned, SOURCE_CACHE, key)
