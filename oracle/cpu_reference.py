"""CPU restatement of the reference's hot-path arithmetic -- TEST INFRASTRUCTURE ONLY.

Not imported by the product. Two restatements live here:

* numpy functions (``matmul_ref`` ... ``rmsnorm_ref``): the algorithms written
  out in float64 from their definitions, independent of torch, used by the
  tests as the checker. Inputs are numpy arrays holding the exact values of
  the low-precision operands (so a bf16 tensor is passed as ``float32`` of its
  values); outputs are float64 arrays, unrounded.
* ``torch_cpu``: the reference's own reference functions (torch ops, on CPU,
  upcast to fp32 as the baseline workload specifies), used as the timed CPU
  baseline in ``bench.py``.

Each function cites the reference code it restates (paths inside the
KernelForge repository, package ``kernelforge``).
"""

from __future__ import annotations

import math

import numpy as np

try:  # scipy's erf is vectorised; math.erf is the fallback
    from scipy.special import erf as _erf
except Exception:  # pragma: no cover
    _erf = np.vectorize(math.erf)

_SQRT_2_OVER_PI = math.sqrt(2.0 / math.pi)


def _f64(a) -> np.ndarray:
    return np.asarray(a, dtype=np.float64)


def matmul_ref(a, b) -> np.ndarray:
    """C = A @ B with exact-as-float64 accumulation.

    Restates ``MatmulOperator.reference`` (kernels/matmul.py:228-233:
    ``torch.matmul`` with TF32 off) and the kernel it gates
    (kernels/matmul.py:54-113: fp32 accumulation of A[m,:]*B[:,n]).
    """
    return _f64(a) @ _f64(b)


def gemv_ref(x, w_nk) -> np.ndarray:
    """Decode-shape Y = X @ W^T with W stored [N, K] (matmul at M in {1,4,16})."""
    return _f64(x) @ _f64(w_nk).T


def gelu_tanh(z) -> np.ndarray:
    """0.5 z (1 + tanh(sqrt(2/pi) (z + 0.044715 z^3)))

    The form ``F.gelu(approximate="tanh")`` computes (kernels/fused_linear.py:16-27,
    160-162); the kernel's sigmoid rewrite (fused_linear.py:22-27, 98-99) is
    the same function.
    """
    z = _f64(z)
    return 0.5 * z * (1.0 + np.tanh(_SQRT_2_OVER_PI * (z + 0.044715 * z * z * z)))


def gelu_erf(z) -> np.ndarray:
    """Exact GELU z * Phi(z) = 0.5 z (1 + erf(z / sqrt 2)) -- the baseline workload's
    form; the reference has no kernel for it, its oracle is ``F.gelu(approximate="none")``."""
    z = _f64(z)
    return 0.5 * z * (1.0 + _erf(z / math.sqrt(2.0)))


def linear_gelu_ref(x, w_kn, bias, approximate: str = "tanh") -> np.ndarray:
    """gelu(x @ w + bias), w in (K, N) orientation.

    Restates ``linear_gelu_reference`` (kernels/fused_linear.py:160-162): the
    unfused matmul, bias add and activation, in that order (the bias is added
    before the activation -- tests/test_fused_linear.py:125-139 pins the order).
    """
    z = _f64(x) @ _f64(w_kn) + _f64(bias)[None, :]
    if approximate == "tanh":
        return gelu_tanh(z)
    if approximate in ("none", "erf"):
        return gelu_erf(z)
    raise ValueError(f"unknown GELU form {approximate!r}")


def softmax_ref(x) -> np.ndarray:
    """Row softmax with the max shift (kernels/softmax.py:1-58, 124-126).

    y = exp(x - max) / sum(exp(x - max)) along the last axis; the shift keeps
    the exponent at or below zero (logits of 60-80 stay finite,
    tests/test_softmax_and_vector_add.py:47-60).
    """
    x = _f64(x)
    shifted = x - x.max(axis=-1, keepdims=True)
    e = np.exp(shifted)
    return e / e.sum(axis=-1, keepdims=True)


def rmsnorm_ref(x, gamma, eps: float = 1e-5) -> np.ndarray:
    """x / sqrt(mean(x^2) + eps) * gamma (kernels/rmsnorm.py:130-143).

    eps inside the square root, so an all-zero row maps to zeros
    (tests/test_rmsnorm.py:110-118). Default eps is the reference's 1e-5.
    """
    x = _f64(x)
    scale = 1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)
    return x * scale * _f64(gamma)[None, :]


class torch_cpu:
    """The reference's own torch reference path on host cores, in fp32.

    These are the functions the reference gates its kernels against
    (matmul.py:228-233, fused_linear.py:160-162, softmax.py:124-126,
    rmsnorm.py:130-143), called on CPU fp32 tensors.
    """

    @staticmethod
    def matmul(a, b):
        import torch

        return torch.matmul(a.float(), b.float())

    @staticmethod
    def linear_gelu(x, w_kn, bias, approximate: str = "tanh"):
        import torch
        import torch.nn.functional as F

        mode = "tanh" if approximate == "tanh" else "none"
        return F.gelu(torch.matmul(x.float(), w_kn.float()) + bias.float(), approximate=mode)

    @staticmethod
    def softmax(x):
        import torch

        return torch.softmax(x.float(), dim=-1)

    @staticmethod
    def rmsnorm(x, gamma, eps: float = 1e-5):
        import torch

        xf = x.float()
        return xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps) * gamma.float()
