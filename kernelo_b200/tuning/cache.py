"""Tuned-configuration cache: the winner of each tuned problem, per device.

The reference keeps its tuned configs in one JSON file nested
``device -> operation -> dtype -> shape`` (``kernelforge/tuning/cache.py:97-129``)
with a version number; that file layout is kept exactly, so a cache written by
either implementation reads in the other.

Inside, the store is a flat index keyed by the 4-tuple (device, operation,
dtype, shape), which the file's nesting is only a serialisation of. Writes are
merges: under an exclusive lock on the cache's directory, the file is re-read,
only the keys this process changed are applied to it, and the result replaces
the file through a temporary file and ``os.replace``. So several tuning
processes (one per GPU, say) can put entries into one cache without losing
each other's, and a crash never leaves a truncated file.

The device part of a key is the board name plus architecture: a file copied to
other hardware misses rather than serving a foreign tuning. Location:
``$KERNELFORGE_CACHE``, else ``$XDG_CACHE_HOME/kernelforge/configs.json``.
"""

from __future__ import annotations

import contextlib
import fcntl
import json
import os
import tempfile
from dataclasses import dataclass
from pathlib import Path

from kernelo_b200.tuning.config import KernelConfig, Problem

CACHE_VERSION = 1

Key = tuple[str, str, str, str]  # (device_key, operation, dtype, shape_key)


def default_cache_path() -> Path:
    if os.environ.get("KERNELFORGE_CACHE"):
        return Path(os.environ["KERNELFORGE_CACHE"])
    root = os.environ.get("XDG_CACHE_HOME") or os.path.join(os.path.expanduser("~"), ".cache")
    return Path(root, "kernelforge", "configs.json")


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
        latency = f"{self.median_us:.1f} us" if self.median_us is not None else "unmeasured"
        params = ", ".join(f"{name}={value}" for name, value in self.config.as_dict().items())
        return (f"{self.device_key}  {self.operation:<16} {self.dtype:<5} {self.shape_key:<22} "
                f"{latency:>12}  {params}")


def _parse(path: Path, text: str) -> dict[Key, dict]:
    """The file's nested document as a flat index (validated)."""
    try:
        doc = json.loads(text)
    except json.JSONDecodeError as exc:
        raise RuntimeError(f"cache file {path} is not valid JSON: {exc}") from exc
    version = doc.get("version") if isinstance(doc, dict) else None
    if version != CACHE_VERSION:
        raise RuntimeError(f"cache file {path} has version {version}, expected {CACHE_VERSION}; "
                           "run `kernelforge cache clear` to discard it")
    index: dict[Key, dict] = {}
    for device, by_op in doc.get("entries", {}).items():
        for operation, by_dtype in by_op.items():
            for dtype, by_shape in by_dtype.items():
                for shape, record in by_shape.items():
                    index[(device, operation, dtype, shape)] = record
    return index


def _document(index: dict[Key, dict]) -> dict:
    """The flat index in the file's nested layout."""
    entries: dict = {}
    for (device, operation, dtype, shape), record in index.items():
        entries.setdefault(device, {}).setdefault(operation, {}).setdefault(dtype, {})[shape] = record
    return {"version": CACHE_VERSION, "entries": entries}


class ConfigCache:
    """Best-known configs in one JSON file (see the module docstring)."""

    def __init__(self, path: str | Path | None = None) -> None:
        self.path = Path(path) if path is not None else default_cache_path()
        self._index: dict[Key, dict] = self._load()

    # ------------------------------------------------------------ file access
    def _load(self) -> dict[Key, dict]:
        try:
            text = self.path.read_text()
        except FileNotFoundError:
            return {}
        return _parse(self.path, text)

    @contextlib.contextmanager
    def _locked(self):
        """Exclusive lock on the cache's directory for a read-merge-write."""
        self.path.parent.mkdir(parents=True, exist_ok=True)
        fd = os.open(self.path.parent, os.O_RDONLY)
        try:
            fcntl.flock(fd, fcntl.LOCK_EX)
            yield
        finally:
            fcntl.flock(fd, fcntl.LOCK_UN)
            os.close(fd)

    def _commit(self, changes: dict[Key, dict]) -> None:
        """Apply ``changes`` to the file as it is now, atomically."""
        with self._locked():
            merged = self._load()
            merged.update(changes)
            fd, tmp = tempfile.mkstemp(dir=self.path.parent, prefix=".configs-", suffix=".tmp")
            try:
                with os.fdopen(fd, "w") as fh:
                    json.dump(_document(merged), fh, indent=2, sort_keys=True)
                    fh.flush()
                    os.fsync(fh.fileno())
                os.replace(tmp, self.path)
            except BaseException:
                with contextlib.suppress(FileNotFoundError):
                    os.unlink(tmp)
                raise
        self._index = merged

    # ------------------------------------------------------------ public API
    @staticmethod
    def _key(problem: Problem, device_key: str) -> Key:
        return (device_key, problem.operation, problem.dtype_name, problem.shape_key)

    def get(self, problem: Problem, device_key: str) -> KernelConfig | None:
        record = self._index.get(self._key(problem, device_key))
        return None if record is None else KernelConfig(problem.operation, **record["config"])

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
        record = {"config": config.as_dict(), "median_us": median_us, "timestamp": timestamp,
                  "candidates_tested": candidates_tested}
        self._commit({self._key(problem, device_key): record})

    def entries(self) -> list[CacheEntry]:
        rows = [
            CacheEntry(device_key=device, operation=operation, dtype=dtype, shape_key=shape,
                       config=KernelConfig(operation, **record["config"]), median_us=record.get("median_us"),
                       timestamp=record.get("timestamp", ""), candidates_tested=record.get("candidates_tested"))
            for (device, operation, dtype, shape), record in self._index.items()
        ]
        return sorted(rows, key=lambda e: (e.device_key, e.operation, e.dtype, e.shape_key))

    def clear(self) -> int:
        removed = len(self._index)
        with self._locked():
            with contextlib.suppress(FileNotFoundError):
                self.path.unlink()
        self._index = {}
        return removed

    def __len__(self) -> int:
        return len(self._index)
