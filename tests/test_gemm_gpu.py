"""GEMM, fused linear and decode GEMV on the B200, against the CPU oracle.

Mirrors the reference's GEMM test strategy (tests/test_matmul.py,
tests/test_fused_linear.py): awkward shapes (primes, one-off-a-tile, single
rows/columns) in every dtype, several tile configs per shape, every budgeted
candidate, non-contiguous views, fp32 held to the fp32 gate, and the fusion's
launch count -- plus the sm_100a specifics: both weight layouts, swapped
skinny shapes, stream-K workspace reuse and determinism, the split tail, the
GELU epilogues held to one ulp of float64, the decode kernels (16-row tiles,
warp-per-row) and the decode-shape fused linear, outputs pre-filled with NaN
so a skipped tile fails, and the baseline's full sizes checked on sampled rows.
"""

from __future__ import annotations

import random

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from kernelo_b200.benchmark import workloads
from kernelo_b200.kernels import gemm_common as gc
from kernelo_b200.kernels.fused_linear import FusedLinearErfOperator, fused_linear_gelu
from kernelo_b200.kernels.gemv import gemv
from kernelo_b200.kernels.matmul import matmul
from kernelo_b200.runtime import native
from kernelo_b200.runtime.env import device_caps
from kernelo_b200.tuning.config import KernelConfig, Problem
from kernelo_b200.tuning.search import FusedLinearSearchSpace, MatmulSearchSpace
from oracle import cpu_reference as ref
from tests.conftest import golden_names, load_golden
from tests.parity import gate, host, sample_rows

pytestmark = pytest.mark.gpu

DTYPES = (torch.float16, torch.bfloat16, torch.float32)
SHAPES = [tuple(p.dims_dict.values()) for p in workloads.problems("matmul", "correctness")]


def operands(m, k, n, dtype, device, seed=0):
    gen = torch.Generator().manual_seed(seed)
    a = torch.randn(m, k, generator=gen).to(dtype).to(device)
    b = torch.randn(k, n, generator=gen).to(dtype).to(device)
    return a, b


def tc(op="matmul", **kw):
    base = dict(KERNEL=1, BLOCK_M=128, BLOCK_N=128, BLOCK_K=64, GROUP_M=8, num_stages=4, STREAM_K=2, SWAP_AB=2)
    base.update(kw)
    return KernelConfig(op, **base)


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("dtype", DTYPES)
def test_matmul_default_config_awkward_shapes(shape, dtype, device):
    m, n, k = shape
    a, b = operands(m, k, n, dtype, device)
    gate(ref.matmul_ref(host(a), host(b)), matmul(a, b), dtype, context=f"{shape} {dtype}")


@pytest.mark.parametrize(
    "config",
    [
        tc(BLOCK_N=64),
        tc(BLOCK_N=128, BLOCK_K=128, num_stages=3),
        tc(BLOCK_N=256, num_stages=3),
        tc(BLOCK_N=128, STREAM_K=1),
        KernelConfig("matmul", KERNEL=2, BLOCK_M=128, BLOCK_N=128, BLOCK_K=8),
        KernelConfig("matmul", KERNEL=2, BLOCK_M=64, BLOCK_N=64, BLOCK_K=16),
    ],
)
@pytest.mark.parametrize("shape", [(127, 192, 64), (257, 256, 512), (1, 128, 4096), (300, 64, 1024)])
def test_matmul_tile_configs_mask_boundaries(config, shape, device):
    m, n, k = shape
    a, b = operands(m, k, n, torch.float16, device)
    gate(ref.matmul_ref(host(a), host(b)), matmul(a, b, config=config), torch.float16,
         context=f"{shape} {config}")


@pytest.mark.parametrize("seed", range(16))
def test_matmul_randomised_shapes_and_candidates(seed, device):
    rng = random.Random(seed)
    m, n, k = (rng.randint(1, 600) for _ in range(3))
    if rng.random() < 0.5:  # half the draws on TMA-friendly multiples of 8
        n, k = 8 * max(1, n // 8), 8 * max(1, k // 8)
    dtype = rng.choice(DTYPES)
    problem = Problem.create("matmul", dtype, M=m, N=n, K=k)
    chosen = rng.choice(MatmulSearchSpace().candidates(problem, device_caps(device)))
    a, b = operands(m, k, n, dtype, device, seed=seed)
    gate(ref.matmul_ref(host(a), host(b)), matmul(a, b, config=chosen), dtype,
         context=f"{m}x{n}x{k} {dtype} {chosen}")


def test_every_budgeted_matmul_candidate_agrees(device):
    problem = Problem.create("matmul", "fp16", M=257, N=512, K=320)
    a, b = operands(257, 320, 512, torch.float16, device)
    expected = ref.matmul_ref(host(a), host(b))
    cands = MatmulSearchSpace().candidates(problem, device_caps(device))
    assert any(c["KERNEL"] == gc.KERNEL_TCGEN05 for c in cands)
    for c in cands:
        gate(expected, matmul(a, b, config=c), torch.float16, context=repr(c))


def test_non_contiguous_views_need_no_copy(device):
    gen = torch.Generator().manual_seed(0)
    for dtype in (torch.float16, torch.bfloat16):
        a = torch.randn(128, 96, generator=gen).to(dtype).to(device).t()   # [96,128], M-major
        b = torch.randn(192, 128, generator=gen).to(dtype).to(device).t()  # [128,192], K-major
        assert not a.is_contiguous() and not b.is_contiguous()
        gate(ref.matmul_ref(host(a), host(b)), matmul(a, b), dtype)
        sliced = torch.randn(64, 256, generator=gen).to(dtype).to(device)[:, 64:192]  # row stride 256
        bb = torch.randn(128, 80, generator=gen).to(dtype).to(device)
        gate(ref.matmul_ref(host(sliced), host(bb)), matmul(sliced, bb), dtype)


def test_fp32_is_ieee_not_tf32(device):
    a, b = operands(512, 1024, 256, torch.float32, device)
    result = gate(ref.matmul_ref(host(a), host(b)), matmul(a, b), torch.float32)
    assert result.error < 1e-5


def test_k_zero_and_empty_outputs(device):
    a = torch.randn(5, 0, device=device, dtype=torch.float16)
    b = torch.randn(0, 7, device=device, dtype=torch.float16)
    assert torch.count_nonzero(matmul(a, b)) == 0
    assert matmul(torch.randn(0, 8, device=device).half(), torch.randn(8, 3, device=device).half()).shape == (0, 3)


def test_matmul_validation(device):
    a = torch.randn(4, 8, device=device, dtype=torch.float16)
    with pytest.raises(ValueError, match="shape mismatch"):
        matmul(a, torch.randn(9, 4, device=device, dtype=torch.float16))
    with pytest.raises(ValueError, match="dtype mismatch"):
        matmul(a, torch.randn(8, 4, device=device, dtype=torch.float32))
    with pytest.raises(ValueError, match="2D"):
        matmul(a, torch.randn(8, device=device, dtype=torch.float16))


def test_infeasible_config_raises_out_of_resources(device):
    a, b = operands(64, 72, 64, torch.float16, device)  # K=72 is fine, N=64 is fine
    with pytest.raises(native.OutOfResources):
        matmul(a, b, config=tc(BLOCK_N=256, BLOCK_K=64, num_stages=8))  # 384 KiB of smem
    c, d = operands(64, 512, 64, torch.float32, device)  # fp32 tiles take 32- or 64-element K blocks
    with pytest.raises(native.OutOfResources, match="BLOCK_K must be 32 or 64"):
        matmul(c, d, config=tc(BLOCK_K=128))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["fp16", "bf16"])
@pytest.mark.parametrize(
    "case",
    ["k509", "n2053", "k3", "odd_base", "transposed_odd", "gather"],
)
def test_unaligned_operands_are_packed_for_tcgen05(case, dtype, device):
    """Operands a TMA tensor map cannot describe -- an odd row pitch along K or
    N, K below one 16-byte vector, a view starting at an odd column, a
    transposed view with an odd pitch, no unit stride at all -- are copied into
    the workspace as pitched matrices and run on tcgen05, by default (M and N
    above 64) and when tcgen05 is asked for at a skinny shape."""
    gen = torch.Generator().manual_seed(7)

    def rnd(*shape):
        return torch.randn(*shape, generator=gen).to(dtype).to(device)

    if case == "k509":
        a, b = rnd(300, 509), rnd(509, 320)
    elif case == "n2053":
        a, b = rnd(257, 512), rnd(512, 2053)
    elif case == "k3":
        a, b = rnd(130, 3), rnd(3, 200)
    elif case == "odd_base":
        a, b = rnd(200, 513)[:, 1:], rnd(512, 264)[:, 3:259]
    elif case == "transposed_odd":
        a, b = rnd(509, 200).t(), rnd(330, 509).t()  # M-major A, K-major B, odd pitches
    else:
        a, b = rnd(400, 300)[::2, ::2], rnd(300, 260)[::2, ::2]  # no unit stride anywhere
    expected = ref.matmul_ref(host(a), host(b))
    out = matmul(a, b)
    gate(expected, out, dtype, context=f"{case} default")
    explicit = tc(BLOCK_N=128, num_stages=3, STREAM_K=2)  # (an N-contiguous B stays MN-major: 64-col boxes)
    gate(expected[:16], matmul(a[:16], b, config=explicit), dtype, context=f"{case} explicit, skinny")


@pytest.mark.parametrize("dtype", DTYPES, ids=lambda d: str(d)[6:])
@pytest.mark.parametrize("m", [1, 2, 3, 5, 8])
def test_column_gemv_row_major_b(m, dtype, device):
    """Up to 8 rows of x against a row-major (K, N) B take the column GEMV (the
    reference's decode layout), every dtype, K split over CTAs with a fixed
    summation order: two calls agree bit for bit."""
    gen = torch.Generator().manual_seed(m)
    x = torch.randn(m, 4096, generator=gen).to(dtype).to(device)
    b = (torch.randn(4096, 11008, generator=gen) * 4096 ** -0.5).to(dtype).to(device)
    assert gc.default_gemm_config("matmul", m, 11008, 4096, dtype, b_layout="kn")["KERNEL"] == gc.KERNEL_COLUMNS
    out = matmul(x, b)
    gate(ref.matmul_ref(host(x), host(b)), out, dtype, context=f"M={m} {dtype}")
    assert torch.equal(out, matmul(x, b)), "deterministic split-K sum"
    # a ragged K (not a multiple of the split) and a strided x
    xs = torch.randn(m, 2 * 1000, generator=gen).to(dtype).to(device)[:, ::2]
    bs = (torch.randn(1000, 4096, generator=gen) * 0.03).to(dtype).to(device)
    gate(ref.matmul_ref(host(xs), host(bs)), matmul(xs, bs), dtype, context=f"M={m} ragged K")


def test_column_gemv_fused_epilogue_and_explicit_config(device):
    """The reference's fused_linear_gelu takes W as (K, N): at decode shapes
    that is the column GEMV with bias + GELU in its final sum."""
    gen = torch.Generator().manual_seed(3)
    x = torch.randn(4, 2048, generator=gen).half().to(device)
    w = (torch.randn(2048, 3072, generator=gen) * 2048 ** -0.5).half().to(device)  # (K, N) row-major
    b = (torch.randn(3072, generator=gen) * 0.3).half().to(device)
    for mode in ("tanh", "none"):
        expected = ref.linear_gelu_ref(host(x), host(w), host(b), mode)
        gate(expected, fused_linear_gelu(x, w, b, approximate=mode), torch.float16, context=mode)
    cols = KernelConfig("matmul", KERNEL=gc.KERNEL_COLUMNS)
    gate(ref.matmul_ref(host(x), host(w)), matmul(x, w, config=cols), torch.float16)
    with pytest.raises(native.OutOfResources):
        matmul(torch.randn(9, 64, device=device).half(), torch.randn(64, 64, device=device).half(), config=cols)


@pytest.mark.parametrize("case", ["odd_n", "odd_column_view"])
def test_output_rows_off_the_16_byte_grid_are_staged(case, device):
    """An output whose rows are off the 16-byte grid (odd N, a view starting at
    an odd column) is written to a pitched copy in the workspace with vector
    stores and moved to C by one copy kernel; columns outside C stay untouched."""
    gen = torch.Generator().manual_seed(5)
    if case == "odd_n":
        a = torch.randn(300, 512, generator=gen).half().to(device)
        w = (torch.randn(1027, 512, generator=gen) * 0.05).half().to(device)  # [N, K], N odd
        bias = torch.randn(1027, generator=gen).half().to(device)
        expected = ref.linear_gelu_ref(host(a), host(w.t()), host(bias), "none")
        gate(expected, fused_linear_gelu(a, w.t(), bias, approximate="none"), torch.float16, context=case)
    else:
        a = torch.randn(256, 512, generator=gen).half().to(device)
        bmat = torch.randn(512, 640, generator=gen).half().to(device)
        full = torch.full((256, 642), 7.0, device=device, dtype=torch.float16)
        out = full[:, 1:641]
        native.gemm(a, bmat, out)
        gate(ref.matmul_ref(host(a), host(bmat)), out, torch.float16, context=case)
        assert torch.all(full[:, 0] == 7.0) and torch.all(full[:, 641] == 7.0)


# ------------------------------------------------------------------ fused linear
def linear_inputs(m, k, n, dtype, device, seed=0, layout="nk"):
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=gen).to(dtype).to(device)
    w = (torch.randn(n, k, generator=gen) * k ** -0.5).to(dtype).to(device)
    b = (torch.randn(n, generator=gen) * 0.316).to(dtype).to(device)
    return x, (w.t() if layout == "nk" else w.t().contiguous()), b


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("approximate", ["tanh", "none"])
def test_fused_linear_matches_unfused_sequence(shape, dtype, approximate, device):
    m, n, k = shape
    x, w, b = linear_inputs(m, k, n, dtype, device)
    expected = ref.linear_gelu_ref(host(x), host(w), host(b), approximate)
    gate(expected, fused_linear_gelu(x, w, b, approximate=approximate), dtype, context=f"{shape} {dtype}")


@pytest.mark.parametrize("layout", ["nk", "kn"])
@pytest.mark.parametrize("m", [1, 16, 100, 513])
def test_fused_linear_weight_layouts_and_skinny_swap(layout, m, device):
    x, w, b = linear_inputs(m, 512, 1000, torch.bfloat16, device, layout=layout)
    gate(ref.linear_gelu_ref(host(x), host(w), host(b), "none"),
         fused_linear_gelu(x, w, b, approximate="none"), torch.bfloat16, context=f"{layout} m={m}")


def test_gelu_over_its_whole_range(device):
    """tests/test_fused_linear.py:96-122 through an identity weight (fp32 -> SIMT path)."""
    g = load_golden("fused_linear_gelu_range_fp32")
    x, w, b = (torch.from_numpy(a).to(device) for a in g["inputs"])
    out = fused_linear_gelu(x, w, b, approximate="tanh")
    assert torch.isfinite(out).all()
    gate(g["ref_torch"], out, torch.float32, threshold=1e-4)
    gate(ref.gelu_tanh(host(x)), out, torch.float32, threshold=1e-4)
    # and the erf form, through bf16 tcgen05 with the identity scaled into range
    xs = torch.linspace(-8, 8, 1024, device=device).reshape(1, -1).bfloat16()
    eye = torch.eye(1024, device=device).bfloat16()
    gate(ref.gelu_erf(host(xs)), fused_linear_gelu(xs, eye, torch.zeros(1024, device=device).bfloat16(),
                                                   approximate="none"), torch.bfloat16)


def test_bias_precedes_activation(device):
    g = load_golden("fused_linear_bias_order_fp32")
    x, w, b = (torch.from_numpy(a).to(device) for a in g["inputs"])
    gate(g["ref_torch"], fused_linear_gelu(x, w, b), torch.float32)
    xb, wb, bb = x.bfloat16(), torch.zeros(32, 64, device=device).bfloat16(), b.bfloat16()
    gate(ref.gelu_tanh(host(bb))[None, :].repeat(8, 0), fused_linear_gelu(xb, wb, bb), torch.bfloat16)


def test_every_budgeted_fused_candidate_agrees(device):
    problem = Problem.create("fused_linear", "fp16", M=257, N=512, K=192)
    x, w, b = linear_inputs(257, 192, 512, torch.float16, device)
    expected = ref.linear_gelu_ref(host(x), host(w), host(b), "tanh")
    for c in FusedLinearSearchSpace().candidates(problem, device_caps(device)):
        gate(expected, fused_linear_gelu(x, w, b, config=c), torch.float16, context=repr(c))


def test_fusion_is_one_launch(device):
    from kernelo_b200.profiling import profile_kernels

    x, w, b = linear_inputs(1024, 1024, 1024, torch.float16, device)
    fused = profile_kernels(lambda: fused_linear_gelu(x, w, b), label="fused", warmup=3, iterations=5)
    unfused = profile_kernels(lambda: F.gelu(x @ w + b, approximate="tanh"), label="unfused",
                              warmup=3, iterations=5)
    assert fused.launches_per_iteration == pytest.approx(1.0, abs=0.01)
    assert unfused.launches_per_iteration >= 2.0


def test_fused_linear_validation(device):
    x = torch.zeros(4, 8, device=device, dtype=torch.float16)
    w = torch.zeros(8, 16, device=device, dtype=torch.float16)
    bias = torch.zeros(16, device=device, dtype=torch.float16)
    with pytest.raises(ValueError, match="bias must have shape"):
        fused_linear_gelu(x, w, torch.zeros(8, device=device, dtype=torch.float16))
    with pytest.raises(ValueError, match="shape mismatch"):
        fused_linear_gelu(x, torch.zeros(9, 16, device=device, dtype=torch.float16), bias)
    with pytest.raises(ValueError, match="dtype mismatch"):
        fused_linear_gelu(x, w.float(), bias)
    with pytest.raises(ValueError, match="approximate"):
        fused_linear_gelu(x, w, bias, approximate="sigmoid")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_baseline_fused_linear_full_size_sampled_rows(dtype, device):
    """4096 x 11008 x 4096, erf GELU, the headline workload: rows checked on a sample."""
    op = FusedLinearErfOperator()
    problem = Problem.create("fused_linear_erf", dtype, M=4096, N=11008, K=4096)
    x, w, b = op.make_inputs(problem, device, seed=0)
    out = op.run(op.default_config(problem), x, w, b)
    rows = sample_rows(4096, 48)
    expected = ref.linear_gelu_ref(host(x[rows]), host(w), host(b), "none")
    gate(expected, out[rows], dtype)
    assert torch.isfinite(out).all()


def test_config0_plain_gemm_full_size_sampled_rows(device):
    """The plain GEMM at its baseline size, 2048 x 4096 x 4096 fp16 with
    row-major (K, N) B, A and B ~ N(0, 1): sampled rows against the float64
    oracle under the fp16 gate, every output finite."""
    from kernelo_b200.kernels.matmul import MatmulOperator

    op = MatmulOperator()
    problem = Problem.create("matmul", "fp16", M=2048, N=4096, K=4096)
    a, b = op.make_inputs(problem, device, seed=0)
    out = op.run(op.default_config(problem), a, b)
    rows = sample_rows(2048, 48)
    gate(ref.matmul_ref(host(a[rows]), host(b)), out[rows], torch.float16, context="2048x4096x4096 fp16")
    assert torch.isfinite(out).all()


SWEEP_SHAPES = [tuple(p.dims_dict.values()) for p in workloads.problems("matmul", "sweep_sm100")]


@pytest.mark.parametrize("shape", SWEEP_SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("dtype", DTYPES, ids=lambda d: str(d)[6:])
def test_tuner_sweep_shapes_every_dtype(shape, dtype, device):
    """The tuner sweep's shapes (primes 4099^3 and 1021x2053x509 whose rows
    TMA cannot describe, one-off-a-tile 129^3 and 257^3, the M=1 decode shape,
    the plain-GEMM baseline) in fp16, bf16 and fp32 on the library default,
    inputs N(0, 1): the oracle on up to 64 sampled rows, fp32 held to 1e-5
    over accumulations up to 4099 long."""
    m, n, k = shape
    a, b = operands(m, k, n, dtype, device, seed=m + n + k)
    out = matmul(a, b)
    rows = sample_rows(m, 64)
    gate(ref.matmul_ref(host(a[rows]), host(b)), out[rows], dtype, context=f"{shape} {dtype}")
    assert torch.isfinite(out).all()


# ------------------------------------------------------------------ golden fixtures
@pytest.mark.parametrize("name", [n for n in golden_names() if n.startswith(("matmul", "fused_linear_"))
                                  and "range" not in n and "bias_order" not in n])
def test_golden_gemm_fixtures(name, device):
    g = load_golden(name)
    dtype = {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32}[g["meta"]["dtype"]]
    ins = [torch.from_numpy(a).to(dtype).to(device) for a in g["inputs"]]
    out = matmul(*ins) if g["meta"]["op"] == "matmul" else fused_linear_gelu(*ins, approximate="tanh")
    gate(g["ref_torch"], out, dtype, context=name)
    if g["ref_kernel"] is not None:
        gate(g["ref_kernel"], out, dtype, context=name + " vs reference kernel")


# ------------------------------------------------------------------ decode GEMV
@pytest.mark.parametrize("m", [1, 4, 16])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("layout", ["nk", "kn"])
def test_gemv_baseline_shapes(m, dtype, layout, device):
    gen = torch.Generator().manual_seed(m)
    x = torch.randn(m, 4096, generator=gen).to(dtype).to(device)
    w_nk = (torch.randn(11008, 4096, generator=gen) * 4096 ** -0.5).to(dtype).to(device)
    w = w_nk if layout == "nk" else w_nk.t().contiguous()
    out = gemv(x, w, w_layout=layout)
    gate(ref.gemv_ref(host(x), host(w_nk)), out, dtype, context=f"M={m} {layout}")


def test_gemv_stream_k_is_deterministic_and_reuses_its_workspace(device):
    """Calls with different tile/grid layouts share one pooled workspace; the
    arrival counters must come back to zero after each, and the fixed-order
    reduction must give bitwise-identical results on repeat."""
    gen = torch.Generator().manual_seed(3)
    x = torch.randn(16, 4096, generator=gen).half().to(device)
    w = (torch.randn(11008, 4096, generator=gen) * 0.02).half().to(device)
    expected = ref.gemv_ref(host(x), host(w))
    first = gemv(x, w)
    for cfg in (
        KernelConfig("gemv", KERNEL=1, BLOCK_M=128, BLOCK_N=16, BLOCK_K=128, num_stages=6, STREAM_K=1, SWAP_AB=1),
        KernelConfig("gemv", KERNEL=1, BLOCK_M=128, BLOCK_N=32, BLOCK_K=64, num_stages=8, STREAM_K=1, SWAP_AB=1,
                     NUM_CTAS=37),
        None,
    ):
        gate(expected, gemv(x, w, config=cfg), torch.float16, context=str(cfg))
    assert torch.equal(first, gemv(x, w))
    assert native.device_status(device.index) == 0


def test_gemv_validation(device):
    x = torch.randn(300, 64, device=device, dtype=torch.float16)
    with pytest.raises(ValueError, match="at most"):
        gemv(x, torch.randn(128, 64, device=device, dtype=torch.float16))
    with pytest.raises(ValueError, match="shape mismatch"):
        gemv(x[:4], torch.randn(128, 65, device=device, dtype=torch.float16))


# ------------------------------------------------------------------ warp-per-row GEMV
WARP_ROWS = KernelConfig("gemv", KERNEL=3)


@pytest.mark.parametrize("m", [1, 2, 3, 4])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_gemv_warp_rows(m, dtype, device):
    """Every compiled row count (1, 2, 4) with unused rows masked; N = 2051 is
    odd (a two-row tile with one row) and leaves the last CTA's warps idle."""
    gen = torch.Generator().manual_seed(10 + m)
    x = torch.randn(m, 1024, generator=gen).to(dtype).to(device)
    w = (torch.randn(2051, 1024, generator=gen) * 1024 ** -0.5).to(dtype).to(device)
    gate(ref.gemv_ref(host(x), host(w)), gemv(x, w, config=WARP_ROWS), dtype, context=f"M={m}")


def test_gemv_warp_rows_tails_and_strides(device):
    """K = 4093 (a 5-element scalar tail after 511 vectors) on weight rows that
    stay 16-byte aligned (row stride 4096), x strided along K, y transposed."""
    gen = torch.Generator().manual_seed(21)
    base = (torch.randn(777, 4096, generator=gen) * 0.02).half().to(device)
    w = base[:, :4093]
    xb = torch.randn(3, 2 * 4093, generator=gen).half().to(device)
    x = xb[:, ::2]
    out = torch.empty(777, 3, device=device, dtype=torch.float16).t()
    gemv(x, w, config=WARP_ROWS, out=out)
    gate(ref.gemv_ref(host(x), host(w)), out, torch.float16)


def test_gemv_warp_rows_refuses_unaligned_weight_rows(device):
    from kernelo_b200.runtime.native import OutOfResources

    x = torch.randn(2, 4097, device=device, dtype=torch.float16)
    w = torch.randn(64, 4097, device=device, dtype=torch.float16)  # rows 8194 bytes apart
    with pytest.raises(OutOfResources, match="16-byte"):
        gemv(x, w, config=WARP_ROWS)
    gate(ref.gemv_ref(host(x), host(w)), gemv(x, w), torch.float16)  # the default falls back


def test_gemv_default_kernel_choice():
    from kernelo_b200.kernels.gemv import default_config

    for m in (1, 2, 4, 16):
        assert default_config(m, 11008, 4096, torch.float16)["KERNEL"] == 4
    assert default_config(1, 11008, 4096, torch.float32)["KERNEL"] == 3
    assert default_config(2, 11008, 4099, torch.bfloat16)["KERNEL"] == 3  # K % 8 != 0
    assert default_config(32, 11008, 4096, torch.float16)["KERNEL"] == 4
    assert default_config(33, 11008, 4096, torch.float16)["KERNEL"] == 1


# ------------------------------------------------------------------ 16-row tile GEMV (mma.sync)
def tile_cfg(warps=0, pairs=0):
    return KernelConfig("gemv", KERNEL=4, BLOCK_M=warps, num_stages=pairs)


@pytest.mark.parametrize("m", [1, 3, 4, 8, 9, 16, 17, 24, 32])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_gemv_tile_rows(m, dtype, device):
    """Both x-row groupings (M <= 8, M <= 16) with unused rows masked; N = 1000
    ends in a half tile; K = 1032 is 129 vectors, so the K slices are uneven
    and the last quad of vectors is partial."""
    gen = torch.Generator().manual_seed(40 + m)
    x = torch.randn(m, 1032, generator=gen).to(dtype).to(device)
    w = (torch.randn(1000, 1032, generator=gen) * 1032 ** -0.5).to(dtype).to(device)
    expected = ref.gemv_ref(host(x), host(w))
    gate(expected, gemv(x, w, config=tile_cfg()), dtype, context=f"M={m} default shape")
    gate(expected, gemv(x, w), dtype, context=f"M={m} library choice")


@pytest.mark.parametrize("shape", [(8, 1), (8, 2), (8, 4), (6, 2), (6, 4), (4, 2), (4, 4), (4, 8)])
@pytest.mark.parametrize("m", [4, 16, 32])
def test_gemv_tile_rows_every_shape(shape, m, device):
    gen = torch.Generator().manual_seed(7 * shape[0] + shape[1])
    x = torch.randn(m, 4096, generator=gen).half().to(device)
    w = (torch.randn(11008, 4096, generator=gen) * 4096 ** -0.5).half().to(device)
    gate(ref.gemv_ref(host(x), host(w)), gemv(x, w, config=tile_cfg(*shape)), torch.float16,
         context=f"shape {shape} M={m}")


@pytest.mark.parametrize("split", [1, 2, 4, 8])
@pytest.mark.parametrize("m,n,k", [(1, 5504, 4096), (16, 1376, 4096), (4, 1000, 1032), (32, 17, 24), (2, 40, 8)])
def test_gemv_tile_rows_split_over_a_cluster(split, m, n, k, device):
    """A weight tile's K extent split over a cluster of 1-8 CTAs (summed in the
    leader's shared memory in rank order): column shards with few tiles, K of
    a single vector (most CTAs of the cluster get no K), ragged N; and the same
    bits whatever the order the CTAs finish in (two runs agree exactly)."""
    gen = torch.Generator().manual_seed(split * 100 + m)
    x = torch.randn(m, k, generator=gen).half().to(device)
    w = (torch.randn(n, k, generator=gen) * k ** -0.5).half().to(device)
    cfg = KernelConfig("gemv", KERNEL=4, BLOCK_M=6 if m > 8 else 8, num_stages=4 if m > 8 else 1, CLUSTER_M=split)
    out = gemv(x, w, config=cfg)
    gate(ref.gemv_ref(host(x), host(w)), out, torch.float16, context=f"split {split} {m}x{n}x{k}")
    assert torch.equal(out, gemv(x, w, config=cfg))


def test_gemv_tile_rows_default_split_fills_the_gpu(device):
    """Few tiles (a column shard) take a K split by default (at least two CTAs
    per SM up to 8 rows of x, four beyond, at most 4 CTAs per tile), and the
    result passes the gate."""
    from kernelo_b200.kernels import gemm_common as gc

    assert gc.tile_rows_split(11008) == 1 and gc.tile_rows_split(5504) == 1 and gc.tile_rows_split(5504, 16) == 2
    assert gc.tile_rows_split(2752) == 2 and gc.tile_rows_split(1376) == 4 and gc.tile_rows_split(1376, 16) == 4
    gen = torch.Generator().manual_seed(3)
    x = torch.randn(4, 4096, generator=gen).half().to(device)
    w = (torch.randn(2752, 4096, generator=gen) * 4096 ** -0.5).half().to(device)
    gate(ref.gemv_ref(host(x), host(w)), gemv(x, w), torch.float16)


def test_gemv_tile_rows_edges_and_strides(device):
    """K of one and two vectors, fewer weight rows than a tile, padded weight and
    x rows (16-byte aligned), y written transposed."""
    gen = torch.Generator().manual_seed(77)
    for n, k in ((5, 8), (16, 16), (17, 24), (33, 264)):
        x = torch.randn(3, k, generator=gen).bfloat16().to(device)
        w = torch.randn(n, k, generator=gen).bfloat16().to(device)
        gate(ref.gemv_ref(host(x), host(w)), gemv(x, w, config=tile_cfg()), torch.bfloat16, context=f"{n}x{k}")
    wb = (torch.randn(300, 1040, generator=gen) * 0.03).half().to(device)
    w = wb[:, :1032]
    xb = torch.randn(12, 1096, generator=gen).half().to(device)
    x = xb[:, :1032]
    out = torch.empty(300, 12, device=device, dtype=torch.float16).t()
    gemv(x, w, config=tile_cfg(), out=out)
    gate(ref.gemv_ref(host(x), host(w)), out, torch.float16)
    assert native.device_status(device.index) == 0


@pytest.mark.parametrize("m", [1, 4, 9, 16])
@pytest.mark.parametrize("approximate", ["tanh", "none"])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_fused_linear_decode_shapes_on_tile_rows(m, approximate, dtype, device):
    """The fused linear at decode shapes (an nn.Linear weight passed as W.t()):
    the library routes it to the 16-row tile kernel with the bias + GELU
    epilogue; the explicit tile config and the tcgen05 path agree with the
    oracle too."""
    from kernelo_b200.kernels.fused_linear import default_config

    gen = torch.Generator().manual_seed(60 + m)
    x = torch.randn(m, 4096, generator=gen).to(dtype).to(device)
    w_nk = (torch.randn(11008, 4096, generator=gen) * 4096 ** -0.5).to(dtype).to(device)
    b = (torch.randn(11008, generator=gen) * 0.3).to(dtype).to(device)
    expected = ref.linear_gelu_ref(host(x), host(w_nk.t()), host(b), approximate)
    cfg = default_config(m, 11008, 4096, dtype)
    assert cfg["KERNEL"] == 4
    for config in (None, cfg, KernelConfig("fused_linear", KERNEL=1)):
        out = fused_linear_gelu(x, w_nk.t(), b, approximate=approximate, config=config)
        gate(expected, out, dtype, context=f"M={m} {approximate} {config}")


def test_tile_rows_bias_only_epilogue_and_plain_matmul(device):
    gen = torch.Generator().manual_seed(5)
    x = torch.randn(3, 1032, generator=gen).half().to(device)
    w_nk = (torch.randn(1000, 1032, generator=gen) * 0.03).half().to(device)
    b = torch.randn(1000, generator=gen).half().to(device)
    y = torch.empty(3, 1000, device=device, dtype=torch.float16)
    native.gemm(x, w_nk.t(), y, bias=b, epilogue=native.KF_EPI_BIAS, launch=native.GemmLaunch())
    gate(ref.matmul_ref(host(x), host(w_nk.t())) + host(b), y, torch.float16, context="bias only")
    gate(ref.matmul_ref(host(x), host(w_nk.t())), matmul(x, w_nk.t()), torch.float16, context="matmul M=3")


def test_gemv_tile_rows_refusals(device):
    from kernelo_b200.runtime.native import OutOfResources

    x = torch.randn(2, 4099, device=device, dtype=torch.float16)
    w = torch.randn(64, 4099, device=device, dtype=torch.float16)
    with pytest.raises(OutOfResources, match="multiple of 8"):
        gemv(x, w, config=tile_cfg())
    gate(ref.gemv_ref(host(x), host(w)), gemv(x, w), torch.float16)  # the library choice falls back
    with pytest.raises(OutOfResources, match="fp16 or bf16"):
        gemv(x[:, :4096].float(), w[:, :4096].float(), config=tile_cfg())
    with pytest.raises((OutOfResources, ValueError)):
        gemv(x[:, :4096], w[:, :4096], config=tile_cfg(5, 3))  # no such compiled shape


@pytest.mark.parametrize("m", [1, 4, 16, 32, 300])
@pytest.mark.parametrize("epilogue", ["none", "erf"])
def test_allgather_peer_stores_on_one_gpu(m, epilogue, device):
    """The all-gathering entry point with "peer" copies that are other buffers
    on this GPU (a peer address is any device pointer): every copy holds the
    block bit for bit, and it equals the plain call's output. M <= 32 runs the
    tile GEMV's peer stores (the decode-shape gather), M = 300 the tcgen05
    epilogue's TMA stores. Y is [M, 2 * 1000] per copy; this call owns columns
    [1000, 2000) of each."""
    gen = torch.Generator().manual_seed(70 + m)
    x = torch.randn(m, 1024, generator=gen).half().to(device)
    w_nk = (torch.randn(1000, 1024, generator=gen) * 0.03).half().to(device)
    b = torch.randn(1000, generator=gen).half().to(device) if epilogue == "erf" else None
    code = native.KF_EPI_BIAS_GELU_ERF if epilogue == "erf" else native.KF_EPI_NONE
    copies = [torch.full((m, 2000), float("nan"), device=device, dtype=torch.float16) for _ in range(3)]
    peers = [c[:, 1000:].data_ptr() for c in copies[1:]]
    native.linear_bias_act_allgather(x, w_nk.t(), copies[0][:, 1000:], peers, bias=b, epilogue=code)
    plain = torch.empty(m, 1000, device=device, dtype=torch.float16)
    native.gemm(x, w_nk.t(), plain, bias=b, epilogue=code, launch=native.GemmLaunch())
    torch.cuda.synchronize()
    for i, c in enumerate(copies):
        assert torch.equal(c[:, 1000:], plain), f"copy {i} differs from the plain call at M={m}"
        assert torch.isnan(c[:, :1000]).all(), f"copy {i}: columns outside the block were written"
    expected = ref.matmul_ref(host(x), host(w_nk.t()))
    if b is not None:
        expected = ref.linear_gelu_ref(host(x), host(w_nk.t()), host(b), "none")
    gate(expected, plain, torch.float16, context=f"M={m} {epilogue}")
    assert native.device_status(device.index or 0) == 0


# ------------------------------------------------------------------ host-buffer fused linear
@pytest.mark.parametrize("m", [1, 300, 1024, 1500])
def test_fused_linear_host_matches_the_oracle(m, device):
    """Row chunks (a partial last chunk, a single chunk, M=1) against the oracle."""
    from kernelo_b200.kernels.fused_linear import fused_linear_gelu_host

    gen = torch.Generator().manual_seed(m)
    x = torch.randn(m, 512, generator=gen).bfloat16()
    w = (torch.randn(768, 512, generator=gen) * 512 ** -0.5).bfloat16().to(device)
    b = (torch.randn(768, generator=gen) * 0.3).bfloat16().to(device)
    out = torch.empty(m, 768, dtype=torch.bfloat16, pin_memory=True)
    got = fused_linear_gelu_host(x.pin_memory(), w.t(), b, approximate="none", out=out, chunks=3)
    torch.cuda.current_stream().synchronize()
    assert got is out
    gate(ref.linear_gelu_ref(host(x), host(w.t()), host(b), "none"), got, torch.bfloat16, context=f"M={m}")


def test_fused_linear_host_validation(device):
    from kernelo_b200.kernels.fused_linear import fused_linear_gelu_host

    w = torch.randn(64, 32, device=device, dtype=torch.bfloat16)
    b = torch.randn(32, device=device, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="pinned"):
        fused_linear_gelu_host(torch.randn(8, 64).bfloat16(), w, b)
    with pytest.raises(ValueError, match="out must be"):
        fused_linear_gelu_host(torch.randn(8, 64).bfloat16().pin_memory(), w, b, out=torch.empty(8, 32).bfloat16())


# ------------------------------------------------------------------ epilogue GELU accuracy
@pytest.mark.parametrize("approximate", ["none", "tanh"])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_epilogue_gelu_within_one_ulp_of_torch(approximate, dtype, device):
    """x = 0 makes the fused output gelu(bias): sweep bias over [-12, 12]
    (negative tail included) and compare each element with GELU evaluated in
    float64 and rounded to the output dtype -- at most one unit in the last
    place apart. The float64 reference avoids the cancellation of 1 + erf and
    1 + tanh in the negative tail (torch's fp32 GELU loses its relative
    accuracy there): 0.5 x erfc(-x / sqrt 2), and x / (1 + exp(-2u))."""
    n = 11008
    bias = torch.linspace(-12, 12, n, device=device).to(dtype)
    x = torch.zeros(128, 64, device=device, dtype=dtype)
    w = torch.randn(n, 64, device=device, dtype=dtype)
    out = fused_linear_gelu(x, w.t(), bias, approximate=approximate)[0].float()
    xd = bias.double()
    if approximate == "tanh":
        u = (2 / torch.pi) ** 0.5 * (xd + 0.044715 * xd ** 3)
        ref64 = xd / (1 + torch.exp(-2 * u))
    else:
        ref64 = 0.5 * xd * torch.special.erfc(-xd / 2 ** 0.5)
    ref = ref64.to(dtype).float()
    mant = 10 if dtype == torch.float16 else 7
    tiny = 2.0 ** (-14 if dtype == torch.float16 else -126)
    ulp = torch.exp2(torch.floor(torch.log2(ref.abs().clamp_min(tiny))) - mant)
    worst = float(((out - ref).abs() / ulp).max())
    assert worst <= 1.0, f"{worst:.2f} ulp"


# ------------------------------------------------------------------ split tail / pair stream-K
def _pair(**kw):
    base = dict(KERNEL=1, BLOCK_M=256, BLOCK_N=256, BLOCK_K=128, num_stages=3, GROUP_M=16, SWAP_AB=2,
                CLUSTER_M=2)
    base.update(kw)
    return KernelConfig("fused_linear_erf", **base)


def _one_sm(**kw):
    base = dict(KERNEL=1, BLOCK_M=128, BLOCK_N=128, BLOCK_K=64, num_stages=6, GROUP_M=8, SWAP_AB=2)
    base.update(kw)
    return KernelConfig("fused_linear_erf", **base)


@pytest.mark.parametrize("shape,cfg", [
    ((4096, 11008, 1024), _pair(STREAM_K=3)),             # 688 pair tiles: 9 waves + 22 tiles as 44 halves
    ((4096, 11008, 1024), _pair(STREAM_K=1)),             # all stream-K on SM pairs
    ((2048, 2816, 2048), _pair(STREAM_K=3, NUM_CTAS=60)),  # 88 tiles on 30 pairs: remainder too large to split
    ((1024, 1024, 4096), _pair(STREAM_K=1)),
    ((1500, 3000, 1000), _pair(STREAM_K=3, BLOCK_N=128, BLOCK_K=64, num_stages=6)),  # ragged edges
    ((2560, 2048, 512), _one_sm(STREAM_K=3)),             # 320 one-SM tiles: 2 waves + 24 as 48 halves
    ((2500, 1990, 512), _one_sm(STREAM_K=3)),             # the same with ragged M and N
])
def test_split_tail_and_pair_stream_k(shape, cfg, device):
    """Whole tiles for the full waves and the last partial wave as half-width
    tiles, or stream-K with the fix-up done per CTA of an SM pair: sampled
    rows against the oracle, bitwise-identical repeats, agreement with whole
    tiles, and a clean device status."""
    m, n, k = shape
    gen = torch.Generator().manual_seed(m + n + k)
    x = torch.randn(m, k, generator=gen).bfloat16().to(device)
    w = (torch.randn(n, k, generator=gen) * k ** -0.5).bfloat16().to(device)
    b = (torch.randn(n, generator=gen) * 0.3).bfloat16().to(device)
    out = fused_linear_gelu(x, w.t(), b, approximate="none", config=cfg)
    rows = sample_rows(m, 48)
    gate(ref.linear_gelu_ref(host(x[rows]), host(w.t()), host(b), "none"), out[rows], torch.bfloat16,
         context=f"{shape} {cfg}")
    assert torch.equal(out, fused_linear_gelu(x, w.t(), b, approximate="none", config=cfg))
    whole = fused_linear_gelu(x, w.t(), b, approximate="none", config=cfg.replace(STREAM_K=2))
    if cfg["STREAM_K"] == 3:  # same K order per output: bitwise the same as whole tiles
        assert torch.equal(out, whole)
    else:
        gate(host(whole[rows].float()), out[rows], torch.bfloat16, context="against whole tiles")
    assert native.device_status(device.index) == 0


def test_split_tail_with_an_mn_major_b(device):
    """matmul's row-major (K, N) B is MN-major: the half-width tiles keep
    64-column TMA boxes."""
    gen = torch.Generator().manual_seed(9)
    a = torch.randn(4096, 1024, generator=gen).half().to(device)
    bm = (torch.randn(1024, 11008, generator=gen) * 1024 ** -0.5).half().to(device)
    cfg = KernelConfig("matmul", KERNEL=1, BLOCK_M=256, BLOCK_N=256, BLOCK_K=128, num_stages=3, GROUP_M=16,
                       SWAP_AB=2, CLUSTER_M=2, STREAM_K=3)
    out = matmul(a, bm, config=cfg)
    rows = sample_rows(4096, 32)
    gate(ref.matmul_ref(host(a[rows]), host(bm)), out[rows], torch.float16)
    assert torch.equal(out, matmul(a, bm, config=cfg.replace(STREAM_K=2)))


def test_auto_stream_k_without_workspace_runs_whole_tiles(device):
    """A C-ABI caller that passes no workspace still gets a result under the
    library's own config: its stream-K choice falls back to whole tiles. An
    explicit stream-K request without workspace is refused."""
    import ctypes

    lib = native.load()
    m, n, k = 4096, 11008, 1024
    gen = torch.Generator().manual_seed(5)
    x = torch.randn(m, k, generator=gen).bfloat16().to(device)
    w = (torch.randn(n, k, generator=gen) * k ** -0.5).bfloat16().to(device)
    b = (torch.randn(n, generator=gen) * 0.3).bfloat16().to(device)
    y = torch.empty(m, n, device=device, dtype=torch.bfloat16)
    wt = w.t()
    stream = torch.cuda.current_stream(device).cuda_stream

    def call(cfg):
        return lib.kf_linear_bias_act(native.native_code(torch.bfloat16), x.data_ptr(), x.stride(0), x.stride(1),
                                      wt.data_ptr(), wt.stride(0), wt.stride(1), b.data_ptr(), y.data_ptr(),
                                      y.stride(0), y.stride(1), m, n, k, native.KF_EPI_BIAS_GELU_ERF,
                                      cfg, None, 0, stream)

    assert call(None) == native.KF_OK
    rows = sample_rows(m, 32)
    gate(ref.linear_gelu_ref(host(x[rows]), host(wt), host(b), "none"), y[rows], torch.bfloat16)
    explicit = native.GemmLaunch.from_config(_pair(STREAM_K=1)).struct()
    assert call(ctypes.byref(explicit)) == native.KF_ERR_WORKSPACE


# ------------------------------------------------------------------ every output written
@pytest.mark.parametrize("case", [
    # (M, N, K, config) through each schedule and kernel: split tail, whole tiles,
    # stream-K on SM pairs and on single SMs, the tile GEMV route, the CUDA-core kernel
    (4096, 11008, 512, None),
    (1000, 3000, 256, KernelConfig("fused_linear", KERNEL=1, STREAM_K=2)),
    (777, 1500, 1024, KernelConfig("fused_linear", KERNEL=1, BLOCK_M=256, STREAM_K=1, CLUSTER_M=2)),
    (300, 700, 384, KernelConfig("fused_linear", KERNEL=1, BLOCK_M=128, STREAM_K=1)),
    (9, 1000, 1032, None),
    (65, 130, 72, KernelConfig("fused_linear", KERNEL=2)),
])
def test_fused_linear_writes_every_output(case, device):
    """The output starts as NaN: a tile the kernel skipped would fail the gate's
    non-finite check (the race-detection plan in place of compute-sanitizer)."""
    m, n, k, config = case
    gen = torch.Generator().manual_seed(m + n)
    x = torch.randn(m, k, generator=gen).bfloat16().to(device)
    w_nk = (torch.randn(n, k, generator=gen) * k ** -0.5).bfloat16().to(device)
    b = (torch.randn(n, generator=gen) * 0.3).bfloat16().to(device)
    out = torch.full((m, n), float("nan"), device=device, dtype=torch.bfloat16)
    fused_linear_gelu(x, w_nk.t(), b, approximate="none", config=config, out=out)
    assert torch.isfinite(out).all(), f"{case}: unwritten outputs"
    rows = torch.arange(0, m, max(1, m // 64))
    gate(ref.linear_gelu_ref(host(x[rows.to(device)]), host(w_nk.t()), host(b), "none"), out[rows.to(device)],
         torch.bfloat16, context=str(case))
    assert native.device_status(device.index) == 0


@pytest.mark.parametrize("m", [1, 3, 16])
@pytest.mark.parametrize("kernel", [1, 3, 4])
def test_gemv_writes_every_output(m, kernel, device):
    if kernel == 3 and m > 4:
        pytest.skip("the warp-per-row kernel takes M <= 4")
    gen = torch.Generator().manual_seed(m * 10 + kernel)
    x = torch.randn(m, 4096, generator=gen).half().to(device)
    w = (torch.randn(5003, 4096, generator=gen) * 4096 ** -0.5).half().to(device)
    out = torch.full((m, 5003), float("nan"), device=device, dtype=torch.float16)
    gemv(x, w, config=KernelConfig("gemv", KERNEL=kernel), out=out)
    assert torch.isfinite(out).all()
    gate(ref.gemv_ref(host(x), host(w)), out, torch.float16, context=f"kernel {kernel} M={m}")
