"""Problem and configuration descriptors (``kernelforge/tuning/config.py:33-150``).

A :class:`KernelConfig` is an immutable, hashable mapping of integer tuning
parameters owned by one operation; each operator's search space defines its
keys. On sm_100a the GEMM keys are ``KERNEL`` (1 = tcgen05, 2 = SIMT),
``BLOCK_M/BLOCK_N/BLOCK_K``, ``GROUP_M``, ``num_stages``, ``STREAM_K``,
``SWAP_AB`` and ``CLUSTER_M/CLUSTER_N``; the row kernels use ``ROW_KERNEL``
(1 = register, 2 = streaming), ``BLOCK_SIZE``, ``num_warps``, and
``ROWS_PER_PROGRAM``/``CLUSTER`` (register kernel) or ``ROW_GROUPS``/``num_stages``
(streaming kernel). All keys travel to the
C ABI; ``meta``/``launch`` keep the reference's split for callers that use it.

A :class:`Problem` is one workload: an operation name, named dimensions in
declaration order and a dtype. Its ``cache_key`` and ``shape_key`` are the
identities used by the config cache and the results database.
"""

from __future__ import annotations

import hashlib
import json
from collections.abc import Iterator, Mapping
from dataclasses import dataclass
from typing import Any

import torch

from kernelo_b200.dtypes import dtype_name, itemsize, parse_dtype

#: Keys the reference passed to Triton's launcher rather than the kernel body.
LAUNCH_KEYS = frozenset({"num_warps", "num_stages"})


class KernelConfig(Mapping[str, int]):
    """Immutable set of integer tuning parameters for one operation."""

    __slots__ = ("operation", "_items")

    def __init__(self, operation: str, **params: int) -> None:
        for key, value in params.items():
            # bool is an int subclass; a True/False parameter is always a bug.
            if isinstance(value, bool) or not isinstance(value, int):
                raise TypeError(f"config parameter {key!r} must be an int, got {value!r}")
        self.operation = operation
        self._items: tuple[tuple[str, int], ...] = tuple(sorted(params.items()))

    # Mapping protocol -------------------------------------------------------
    def __getitem__(self, key: str) -> int:
        for k, v in self._items:
            if k == key:
                return v
        raise KeyError(key)

    def __iter__(self) -> Iterator[str]:
        return (k for k, _ in self._items)

    def __len__(self) -> int:
        return len(self._items)

    def __hash__(self) -> int:
        return hash((self.operation, self._items))

    def __eq__(self, other: object) -> bool:
        if not isinstance(other, KernelConfig):
            return NotImplemented
        return (self.operation, self._items) == (other.operation, other._items)

    def __repr__(self) -> str:
        inner = ", ".join(f"{k}={v}" for k, v in self._items)
        return f"KernelConfig({self.operation!r}, {inner})"

    # Views ------------------------------------------------------------------
    @property
    def meta(self) -> dict[str, int]:
        return {k: v for k, v in self._items if k not in LAUNCH_KEYS}

    @property
    def launch(self) -> dict[str, int]:
        return {k: v for k, v in self._items if k in LAUNCH_KEYS}

    def as_dict(self) -> dict[str, int]:
        return dict(self._items)

    def replace(self, **changes: int) -> KernelConfig:
        merged = self.as_dict()
        merged.update(changes)
        return KernelConfig(self.operation, **merged)

    def to_json(self) -> str:
        return json.dumps(self.as_dict(), sort_keys=True, separators=(",", ":"))

    @classmethod
    def from_json(cls, operation: str, payload: str) -> KernelConfig:
        return cls(operation, **json.loads(payload))

    @property
    def digest(self) -> str:
        """16-hex-digit content hash; the database identity of a config."""
        blob = (self.operation + "|" + self.to_json()).encode()
        return hashlib.sha1(blob).hexdigest()[:16]

    def render(self, order: tuple[str, ...] = ()) -> str:
        """One ``key: value`` line per parameter, ``order`` first."""
        keys = [k for k in order if k in self] + [k for k in self if k not in order]
        width = max((len(k) for k in keys), default=0) + 1
        return "\n".join(f"{(k + ':'):<{width}} {self[k]:>4}" for k in keys)


@dataclass(frozen=True)
class Problem:
    """One workload: an operation at named dimensions and a dtype."""

    operation: str
    dims: tuple[tuple[str, int], ...]
    dtype: torch.dtype

    @classmethod
    def create(cls, operation: str, dtype: str | torch.dtype, **dims: int) -> Problem:
        for name, value in dims.items():
            if isinstance(value, bool) or not isinstance(value, int) or value < 1:
                raise ValueError(f"dimension {name!r} must be a positive int, got {value!r}")
        return cls(operation, tuple(dims.items()), parse_dtype(dtype))

    def __getitem__(self, key: str) -> int:
        return self.dims_dict[key]

    @property
    def dims_dict(self) -> dict[str, int]:
        return dict(self.dims)

    @property
    def shape_key(self) -> str:
        return "x".join(str(v) for _, v in self.dims)

    @property
    def dtype_name(self) -> str:
        return dtype_name(self.dtype)

    @property
    def itemsize(self) -> int:
        return itemsize(self.dtype)

    @property
    def cache_key(self) -> str:
        return f"{self.operation}/{self.dtype_name}/{self.shape_key}"

    def describe(self) -> str:
        names = "/".join(k for k, _ in self.dims)
        values = " x ".join(str(v) for _, v in self.dims)
        return f"{self.operation} {names}={values} {self.dtype_name}"

    def as_dict(self) -> dict[str, Any]:
        return {
            "operation": self.operation,
            "dims": self.dims_dict,
            "dtype": self.dtype_name,
            "shape_key": self.shape_key,
        }
