"""The CPU oracle, pinned against the reference (no GPU needed).

Every fixture in ``tests/golden`` was produced by the reference's own code:
its gate references in the operand dtype (``ref_torch``) and, for fp16/fp32,
its Triton kernels run under the Triton interpreter (``ref_kernel``). The
oracle must agree with both under the reference's own gate (testing.py:31-35),
and must reproduce the reference tests' known-answer pins.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from kernelo_b200.testing import threshold_for, verify
from oracle import cpu_reference as ref
from tests.conftest import golden_names, load_golden

DTYPES = {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32}


def oracle_for(g: dict) -> np.ndarray:
    meta, ins = g["meta"], g["inputs"]
    op = meta["op"]
    if op == "matmul":
        return ref.matmul_ref(*ins)
    if op == "fused_linear":
        return ref.linear_gelu_ref(*ins, approximate=meta.get("approximate", "tanh"))
    if op == "softmax":
        return ref.softmax_ref(*ins)
    if op == "rmsnorm":
        return ref.rmsnorm_ref(*ins, eps=meta["eps"])
    raise AssertionError(op)


@pytest.mark.parametrize("name", golden_names())
def test_oracle_matches_reference_gate_reference(name):
    g = load_golden(name)
    dtype = DTYPES[g["meta"]["dtype"]]
    expected = torch.from_numpy(g["ref_torch"])
    got = torch.from_numpy(oracle_for(g)).float()
    result = verify(expected, got, dtype=dtype)
    assert result.passed, f"{name}: {result.reason}"


@pytest.mark.parametrize("name", [n for n in golden_names() if load_golden(n)["ref_kernel"] is not None])
def test_oracle_matches_reference_triton_kernel(name):
    g = load_golden(name)
    dtype = DTYPES[g["meta"]["dtype"]]
    expected = torch.from_numpy(g["ref_kernel"])
    got = torch.from_numpy(oracle_for(g)).float()
    # The interpreter's fp32 tl.dot is IEEE; fp16 kernels round once at the end.
    result = verify(got, expected, dtype=dtype)
    assert result.passed, f"{name}: {result.reason}"


def test_fixture_set_covers_every_operator_and_dtype():
    seen = {(load_golden(n)["meta"]["op"], load_golden(n)["meta"]["dtype"]) for n in golden_names()}
    for op in ("matmul", "fused_linear", "softmax", "rmsnorm"):
        for dt in ("fp16", "bf16", "fp32"):
            assert (op, dt) in seen, (op, dt)


# ---- known-answer pins from the reference's tests -------------------------
def test_gelu_tanh_range_and_tails():
    """tests/test_fused_linear.py:96-122: finite everywhere, correct limits."""
    z = np.concatenate([np.linspace(-60, 60, 512), [-1e4, -100, -1e-7, 0, 1e-7, 100, 1e4]])
    y = ref.gelu_tanh(z)
    assert np.isfinite(y).all()
    assert y[-7] == 0.0 and y[-1] == 1e4  # large negative -> 0, large positive -> identity
    expected = torch.nn.functional.gelu(torch.from_numpy(z), approximate="tanh").numpy()
    assert np.max(np.abs(y - expected)) / np.max(np.abs(expected)) < 1e-12


def test_gelu_erf_matches_torch_exact_gelu():
    z = np.linspace(-12, 12, 4001)
    expected = torch.nn.functional.gelu(torch.from_numpy(z), approximate="none").numpy()
    assert np.max(np.abs(ref.gelu_erf(z) - expected)) < 1e-12


def test_bias_is_added_before_the_activation():
    """tests/test_fused_linear.py:125-139: zero W -> gelu(bias) in every row."""
    x = np.random.default_rng(0).standard_normal((8, 32))
    bias = np.linspace(-4, 4, 64)
    out = ref.linear_gelu_ref(x, np.zeros((32, 64)), bias)
    assert np.allclose(out, ref.gelu_tanh(bias)[None, :].repeat(8, 0))


def test_softmax_constant_row_is_exactly_uniform():
    """tests/test_softmax_and_vector_add.py:63-69."""
    out = ref.softmax_ref(np.full((2, 128), -3.5))
    assert np.all(out == 1.0 / 128)


def test_softmax_overflowing_logits_stay_finite():
    """tests/test_softmax_and_vector_add.py:47-60: logits 60/80 sum to one."""
    x = np.full((4, 512), 60.0)
    x[:, 0] = 80.0
    out = ref.softmax_ref(x)
    assert np.isfinite(out).all()
    assert np.allclose(out.sum(-1), 1.0)


def test_rmsnorm_zero_row_is_finite():
    """tests/test_rmsnorm.py:110-118: eps inside the square root."""
    assert np.all(ref.rmsnorm_ref(np.zeros((4, 256)), np.ones(256)) == 0.0)


def test_rmsnorm_needs_the_wide_reduction():
    """tests/test_rmsnorm.py:79-107: an fp16 running sum is visibly worse."""
    rng = np.random.default_rng(0)
    x = rng.standard_normal((64, 8192)).astype(np.float16).astype(np.float32)
    gamma = (rng.standard_normal(8192) * 0.1 + 1).astype(np.float16).astype(np.float32)
    exact = ref.rmsnorm_ref(x, gamma)
    naive_sum = np.zeros((64, 1), dtype=np.float16)
    for j in range(0, 8192, 512):  # blocked fp16 accumulation
        naive_sum = (naive_sum + (x[:, j:j + 512] ** 2).sum(-1, keepdims=True).astype(np.float16)).astype(np.float16)
    naive = x / np.sqrt(naive_sum.astype(np.float64) / 8192 + 1e-5) * gamma
    err = np.max(np.abs(naive - exact)) / np.max(np.abs(exact))
    assert err > 1e-4


def test_thresholds_are_the_references():
    assert threshold_for(torch.float32) == 1e-5
    assert threshold_for(torch.float16) == 5e-3
    assert threshold_for(torch.bfloat16) == 2e-2


def test_torch_cpu_baseline_agrees_with_numpy_oracle():
    gen = torch.Generator().manual_seed(1)
    x = torch.randn(16, 64, generator=gen)
    w = torch.randn(64, 32, generator=gen) * 0.125
    b = torch.randn(32, generator=gen)
    for mode in ("tanh", "none"):
        a = ref.torch_cpu.linear_gelu(x, w, b, mode).numpy()
        e = ref.linear_gelu_ref(x.numpy(), w.numpy(), b.numpy(), mode)
        assert np.max(np.abs(a - e)) < 1e-5
    assert np.max(np.abs(ref.torch_cpu.softmax(x).numpy() - ref.softmax_ref(x.numpy()))) < 1e-6
    g = torch.ones(64)
    assert np.max(np.abs(ref.torch_cpu.rmsnorm(x, g).numpy() - ref.rmsnorm_ref(x.numpy(), g.numpy()))) < 1e-5
