"""Tuned-configuration cache (``kernelforge/tuning/cache.py:1-159``).

A JSON file nested ``device -> operation -> dtype -> shape`` holding the winning
config of each tuned problem, so a serving process reads a tuning instead of
re-running it. The device part is the board name plus architecture: a file
copied to other hardware misses rather than serving a foreign tuning. Writes
go through a temporary file and ``os.replace`` so a crash never leaves a
truncated cache. Location: ``$KERNELFORGE_CACHE``, else
``$XDG_CACHE_HOME/kernelforge/configs.json``.
"""

from __future__ import annotations

import json
import os
import tempfile
from dataclasses import dataclass
from pathlib import Path
from typing import Any

from kernelo_b200.tuning.config import KernelConfig, Problem

CACHE_VERSION = 1


def default_cache_path() -> Path:
    explicit = os.environ.get("KERNELFORGE_CACHE")
    if explicit:
        return Path(explicit)
    base = Path(os.environ.get("XDG_CACHE_HOME", str(Path.home() / ".cache")))
    return base / "kernelforge" / "configs.json"


@dataclass(frozen=True)
class CacheEntry:
    device_key: str
    operation: str
    dtype: str
    shape_key: str
    config: KernelConfig
    median_us: float | None
    timestamp: str
    candidates_tested: int | None = None

    def describe(self) -> str:
        params = ", ".join(f"{k}={v}" for k, v in self.config.as_dict().items())
        latency = "unmeasured" if self.median_us is None else f"{self.median_us:.1f} us"
        return (
            f"{self.device_key}  {self.operation:<16} {self.dtype:<5} "
            f"{self.shape_key:<22} {latency:>12}  {params}"
        )


class ConfigCache:
    """Best-known configs in one JSON file."""

    def __init__(self, path: str | Path | None = None) -> None:
        self.path = Path(path) if path is not None else default_cache_path()
        self._data = self._read()

    def _read(self) -> dict[str, Any]:
        if not self.path.exists():
            return {"version": CACHE_VERSION, "entries": {}}
        try:
            data = json.loads(self.path.read_text())
        except json.JSONDecodeError as exc:
            raise RuntimeError(f"cache file {self.path} is not valid JSON: {exc}") from exc
        if data.get("version") != CACHE_VERSION:
            raise RuntimeError(
                f"cache file {self.path} has version {data.get('version')}, expected "
                f"{CACHE_VERSION}; run `kernelforge cache clear` to discard it"
            )
        return data

    def _write(self) -> None:
        self.path.parent.mkdir(parents=True, exist_ok=True)
        fd, tmp_name = tempfile.mkstemp(dir=self.path.parent, suffix=".tmp")
        try:
            with os.fdopen(fd, "w") as fh:
                json.dump(self._data, fh, indent=2, sort_keys=True)
            os.replace(tmp_name, self.path)
        except BaseException:
            Path(tmp_name).unlink(missing_ok=True)
            raise

    def _node(self, device_key: str, problem: Problem, *, create: bool) -> dict[str, Any] | None:
        node: dict[str, Any] = self._data["entries"]
        for key in (device_key, problem.operation, problem.dtype_name):
            if key not in node:
                if not create:
                    return None
                node[key] = {}
            node = node[key]
        return node

    def get(self, problem: Problem, device_key: str) -> KernelConfig | None:
        node = self._node(device_key, problem, create=False)
        if node is None or problem.shape_key not in node:
            return None
        return KernelConfig(problem.operation, **node[problem.shape_key]["config"])

    def put(
        self,
        problem: Problem,
        device_key: str,
        config: KernelConfig,
        *,
        median_us: float | None = None,
        timestamp: str = "",
        candidates_tested: int | None = None,
    ) -> None:
        node = self._node(device_key, problem, create=True)
        assert node is not None
        node[problem.shape_key] = {
            "config": config.as_dict(),
            "median_us": median_us,
            "timestamp": timestamp,
            "candidates_tested": candidates_tested,
        }
        self._write()

    def entries(self) -> list[CacheEntry]:
        found = []
        for device_key, ops in self._data["entries"].items():
            for operation, dtypes in ops.items():
                for dtype, shapes in dtypes.items():
                    for shape_key, payload in shapes.items():
                        found.append(
                            CacheEntry(
                                device_key=device_key,
                                operation=operation,
                                dtype=dtype,
                                shape_key=shape_key,
                                config=KernelConfig(operation, **payload["config"]),
                                median_us=payload.get("median_us"),
                                timestamp=payload.get("timestamp", ""),
                                candidates_tested=payload.get("candidates_tested"),
                            )
                        )
        found.sort(key=lambda e: (e.device_key, e.operation, e.dtype, e.shape_key))
        return found

    def clear(self) -> int:
        count = len(self.entries())
        self._data = {"version": CACHE_VERSION, "entries": {}}
        if self.path.exists():
            self.path.unlink()
        return count

    def __len__(self) -> int:
        return len(self.entries())
