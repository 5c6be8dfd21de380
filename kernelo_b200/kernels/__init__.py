"""Operator registry (``kernelforge/kernels/__init__.py:17-38``).

Operators resolve lazily by name, so ``import kernelo_b200`` never loads the
native library; it is loaded (and built if needed) on the first kernel call.
"""

from __future__ import annotations

import importlib
from typing import TYPE_CHECKING

if TYPE_CHECKING:
    from kernelo_b200.kernels.base import Operator

_OPERATORS: dict[str, tuple[str, str]] = {
    "softmax": ("kernelo_b200.kernels.softmax", "SoftmaxOperator"),
    "matmul": ("kernelo_b200.kernels.matmul", "MatmulOperator"),
    "rmsnorm": ("kernelo_b200.kernels.rmsnorm", "RMSNormOperator"),
    "fused_linear": ("kernelo_b200.kernels.fused_linear", "FusedLinearOperator"),
    "fused_linear_erf": ("kernelo_b200.kernels.fused_linear", "FusedLinearErfOperator"),
    "gemv": ("kernelo_b200.kernels.gemv", "GemvOperator"),
}


def operator_names() -> tuple[str, ...]:
    return tuple(_OPERATORS)


def get_operator(name: str, **kwargs) -> Operator:
    try:
        module_path, class_name = _OPERATORS[name]
    except KeyError:
        raise ValueError(
            f"unknown operator {name!r}; available: {', '.join(operator_names())}"
        ) from None
    return getattr(importlib.import_module(module_path), class_name)(**kwargs)
