"""Softmax and RMSNorm on the B200 against the CPU oracle.

Follows tests/test_softmax_and_vector_add.py and tests/test_rmsnorm.py of the
reference: awkward widths in every dtype, overflow logits, constant rows, zero
rows, the fp32-reduction teeth test, indivisible rows per program, every
candidate -- plus the widths the reference kernels refuse (4097 with unaligned
rows, 32000 through a thread-block cluster), the streaming kernel's launch
shapes and refusals, the kernel chosen per row width, outputs pre-filled with
NaN, and the baseline sizes.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from kernelo_b200.benchmark import workloads
from kernelo_b200.kernels.rmsnorm import RMSNormOperator, rmsnorm
from kernelo_b200.kernels.softmax import SoftmaxOperator, softmax
from kernelo_b200.runtime.env import device_caps
from kernelo_b200.tuning.config import KernelConfig, Problem
from kernelo_b200.tuning.search import RMSNormSearchSpace, SoftmaxSearchSpace
from oracle import cpu_reference as ref
from tests.conftest import golden_names, load_golden
from tests.parity import gate, host, sample_rows

pytestmark = pytest.mark.gpu

DTYPES = (torch.float16, torch.bfloat16, torch.float32)
ROW_SHAPES = [tuple(p.dims_dict.values()) for p in workloads.problems("softmax", "correctness")] + [
    (8, 4097), (4, 32000), (2, 65536), (3, 1000)]


def rand(rows, cols, dtype, device, scale=1.0, seed=0):
    gen = torch.Generator().manual_seed(seed)
    return (torch.randn(rows, cols, generator=gen) * scale).to(dtype).to(device)


@pytest.mark.parametrize("shape", ROW_SHAPES)
@pytest.mark.parametrize("dtype", DTYPES)
def test_softmax_shapes(shape, dtype, device):
    x = rand(*shape, dtype, device, scale=4.0)
    gate(ref.softmax_ref(host(x)), softmax(x), dtype, context=f"{shape}")


@pytest.mark.parametrize("shape", ROW_SHAPES)
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("eps", [1e-5, 1e-6])
def test_rmsnorm_shapes(shape, dtype, eps, device):
    x = rand(*shape, dtype, device)
    gamma = (rand(1, shape[1], torch.float32, device, seed=1)[0] * 0.1 + 1).to(dtype)
    gate(ref.rmsnorm_ref(host(x), host(gamma), eps), rmsnorm(x, gamma, eps=eps), dtype, context=f"{shape}")


def test_softmax_logits_that_overflow_fp16(device):
    x = torch.full((4, 512), 60.0, device=device, dtype=torch.float16)
    x[:, 0] = 80.0
    out = softmax(x)
    assert torch.isfinite(out).all()
    gate(ref.softmax_ref(host(x)), out, torch.float16)
    assert torch.allclose(out.float().sum(-1), torch.ones(4, device=device), atol=1e-2)


def test_softmax_constant_row_is_uniform(device):
    out = softmax(torch.full((2, 128), -3.5, device=device))
    assert torch.allclose(out, torch.full_like(out, 1 / 128), atol=1e-6)


def test_rmsnorm_zero_row_is_finite(device):
    out = rmsnorm(torch.zeros(4, 256, device=device, dtype=torch.float16),
                  torch.ones(256, device=device, dtype=torch.float16))
    assert torch.isfinite(out).all() and torch.count_nonzero(out) == 0


def test_wide_fp16_rows_need_the_fp32_reduction(device):
    x = rand(64, 8192, torch.float16, device)
    gamma = (rand(1, 8192, torch.float32, device, seed=1)[0] * 0.1 + 1).half()
    result = gate(ref.rmsnorm_ref(host(x), host(gamma)), rmsnorm(x, gamma), torch.float16)
    naive_sum = x.pow(2).sum(-1, keepdim=True, dtype=torch.float16)
    naive = (x * torch.rsqrt(naive_sum.float() / 8192 + 1e-5) * gamma).half()
    from kernelo_b200.testing import verify

    assert verify(torch.from_numpy(ref.rmsnorm_ref(host(x), host(gamma))), naive.cpu().double(),
                  dtype=torch.float16).error > result.error


@pytest.mark.parametrize("rows_per_program", [1, 2, 4, 8])
@pytest.mark.parametrize("rows", [1, 3, 7, 17, 129])
def test_rows_per_program_with_indivisible_rows(rows_per_program, rows, device):
    x = rand(rows, 513, torch.float16, device)
    gamma = torch.ones(513, device=device, dtype=torch.float16)
    cfg = KernelConfig("rmsnorm", BLOCK_SIZE=1024, ROWS_PER_PROGRAM=rows_per_program, num_warps=2, CLUSTER=1)
    gate(ref.rmsnorm_ref(host(x), host(gamma)), rmsnorm(x, gamma, config=cfg), torch.float16)
    cfg = KernelConfig("softmax", BLOCK_SIZE=1024, ROWS_PER_PROGRAM=rows_per_program, num_warps=2, CLUSTER=2)
    gate(ref.softmax_ref(host(x)), softmax(x, config=cfg), torch.float16)


def test_every_candidate_agrees(device):
    for space, fn, name in ((SoftmaxSearchSpace(), softmax, "softmax"), (RMSNormSearchSpace(), None, "rmsnorm")):
        problem = Problem.create(name, "fp16", rows=333, cols=2048)
        x = rand(333, 2048, torch.float16, device)
        gamma = torch.ones(2048, device=device, dtype=torch.float16)
        expected = ref.softmax_ref(host(x)) if name == "softmax" else ref.rmsnorm_ref(host(x), host(gamma))
        for c in space.candidates(problem, device_caps(device)):
            out = softmax(x, config=c) if name == "softmax" else rmsnorm(x, gamma, config=c)
            gate(expected, out, torch.float16, context=repr(c))


def test_row_strided_input(device):
    base = rand(64, 1536, torch.bfloat16, device)
    x = base[:, 256:1280]  # row stride 1536, last dim contiguous
    gate(ref.softmax_ref(host(x)), softmax(x), torch.bfloat16)
    gamma = torch.ones(1024, device=device, dtype=torch.bfloat16)
    gate(ref.rmsnorm_ref(host(x), host(gamma)), rmsnorm(x, gamma), torch.bfloat16)


def test_validation(device):
    with pytest.raises(ValueError, match="2D"):
        softmax(torch.zeros(2, 3, 4, device=device, dtype=torch.float16))
    with pytest.raises(ValueError, match="contiguous"):
        softmax(torch.zeros(8, 8, device=device).t())
    with pytest.raises(ValueError, match="gamma must have shape"):
        rmsnorm(torch.zeros(4, 128, device=device), torch.ones(64, device=device))
    cfg = KernelConfig("rmsnorm", BLOCK_SIZE=256, ROWS_PER_PROGRAM=1, num_warps=4, CLUSTER=1)
    with pytest.raises(ValueError, match="cannot hold a row"):
        rmsnorm(torch.zeros(8, 1024, device=device), torch.ones(1024, device=device), config=cfg)
    with pytest.raises(ValueError, match="single-pass limit"):
        softmax(torch.zeros(1, 300_000, device=device, dtype=torch.float16))


@pytest.mark.parametrize("name", [n for n in golden_names() if n.startswith(("softmax", "rmsnorm"))])
def test_golden_row_fixtures(name, device):
    g = load_golden(name)
    meta = g["meta"]
    dtype = {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32}[meta["dtype"]]
    ins = [torch.from_numpy(a).to(dtype).to(device) for a in g["inputs"]]
    out = softmax(ins[0]) if meta["op"] == "softmax" else rmsnorm(*ins, eps=meta["eps"])
    gate(g["ref_torch"], out, dtype, context=name)
    if g["ref_kernel"] is not None:
        gate(g["ref_kernel"], out, dtype, context=name + " vs reference kernel")


# ---------------------------------------------------------------- baseline sizes
@pytest.mark.parametrize("cols", [1000, 4096, 4097, 32000])
@pytest.mark.parametrize("dtype", DTYPES, ids=lambda d: str(d)[6:])
def test_softmax_baseline_sizes(cols, dtype, device):
    """[32768, C] with x ~ N(0, 4^2), every width and dtype of the baseline:
    sampled rows against the oracle, every row sums to 1."""
    op = SoftmaxOperator()
    problem = Problem.create("softmax", dtype, rows=32768, cols=cols)
    (x,) = op.make_inputs(problem, device)
    out = softmax(x)
    rows = sample_rows(32768, 32)
    gate(ref.softmax_ref(host(x[rows])), out[rows], dtype)
    sums = out.float().sum(-1)
    tol = {torch.float32: 1e-4, torch.bfloat16: 0.05, torch.float16: 0.01}[dtype]
    assert float((sums - 1).abs().max()) < tol


@pytest.mark.parametrize("cols", [4096, 8192])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_rmsnorm_baseline_sizes(cols, dtype, device):
    op = RMSNormOperator(eps=1e-6)
    problem = Problem.create("rmsnorm", dtype, rows=16384, cols=cols)
    x, gamma = op.make_inputs(problem, device)
    out = op.run(op.default_config(problem), x, gamma)
    rows = sample_rows(16384, 32)
    gate(ref.rmsnorm_ref(host(x[rows]), host(gamma), 1e-6), out[rows], dtype)
    # Normalised rows have unit RMS before gamma: undo gamma and check.
    rms = (out.float() / gamma.float()).pow(2).mean(-1).sqrt()
    assert float((rms - 1).abs().max()) < (0.02 if dtype == torch.bfloat16 else 0.005)


# ---------------------------------------------------------------- streaming kernel
def stream_cfg(op, cols, **kw):
    return KernelConfig(op, BLOCK_SIZE=max(1, 1 << (cols - 1).bit_length()), ROW_KERNEL=2, **kw)


STREAM_COLS = (1, 3, 8, 9, 127, 1000, 2048, 4097, 8192, 16000, 32000)


@pytest.mark.parametrize("cols", STREAM_COLS)
@pytest.mark.parametrize("dtype", DTYPES)
def test_stream_kernel_widths(cols, dtype, device):
    """Explicit streaming kernel at its default warps: widths below one vector,
    unaligned (4097) rows with scalar head/tail, up to 64-128 KiB rows."""
    from kernelo_b200.kernels.rows_common import stream_default_warps

    rows = 2 * 148 + 5
    x = rand(rows, cols, dtype, device, scale=4.0)
    warps = stream_default_warps(cols, dtype)
    gate(ref.softmax_ref(host(x)), softmax(x, config=stream_cfg("softmax", cols, num_warps=warps)), dtype,
         context=f"softmax {cols}")
    gamma = (rand(1, cols, torch.float32, device, seed=1)[0] * 0.1 + 1).to(dtype)
    x1 = rand(rows, cols, dtype, device)
    gate(ref.rmsnorm_ref(host(x1), host(gamma), 1e-6),
         rmsnorm(x1, gamma, eps=1e-6, config=stream_cfg("rmsnorm", cols, num_warps=warps)), dtype,
         context=f"rmsnorm {cols}")


@pytest.mark.parametrize("warps", [1, 2, 4, 8, 16])
@pytest.mark.parametrize("row_groups,stages", [(0, 0), (1, 0), (3, 0), (0, 1), (0, 2), (2, 5)])
def test_stream_kernel_launch_shapes(warps, row_groups, stages, device):
    """Every warps x row-group x ring-depth combination, including one slot
    shared by all groups (stages=1) and more groups than slots."""
    if row_groups * warps > 16:
        pytest.skip("more than 16 consumer warps")
    x = rand(1000, 2048, torch.float16, device, scale=4.0)
    gamma = (rand(1, 2048, torch.float32, device, seed=1)[0] * 0.1 + 1).half()
    kw = dict(num_warps=warps, ROW_GROUPS=row_groups, num_stages=stages)
    gate(ref.softmax_ref(host(x)), softmax(x, config=stream_cfg("softmax", 2048, **kw)), torch.float16)
    gate(ref.rmsnorm_ref(host(x), host(gamma)), rmsnorm(x, gamma, config=stream_cfg("rmsnorm", 2048, **kw)),
         torch.float16)


def test_stream_kernel_sixteen_vectors_per_thread(device):
    """The 16-vector instantiation (rows of 128 KiB fp32 / 64 KiB 16-bit at 16 warps)."""
    for dtype, cols in ((torch.float32, 32000), (torch.bfloat16, 64000)):
        x = rand(300, cols, dtype, device, scale=4.0)
        gate(ref.softmax_ref(host(x)), softmax(x, config=stream_cfg("softmax", cols, num_warps=16)), dtype,
             context=f"{dtype} {cols}")


def test_stream_kernel_strided_rows(device):
    base = rand(600, 1536, torch.bfloat16, device, scale=4.0)
    x = base[:, 8:1008]  # row stride 1536, 16-byte-aligned start: same phase as the output
    out = softmax(x, config=stream_cfg("softmax", 1000, num_warps=1))
    gate(ref.softmax_ref(host(x)), out, torch.bfloat16)
    gamma = torch.ones(1000, device=device, dtype=torch.bfloat16)
    gate(ref.rmsnorm_ref(host(x), host(gamma)), rmsnorm(x, gamma, config=stream_cfg("rmsnorm", 1000, num_warps=1)),
         torch.bfloat16)
    # A start off the 16-byte grid puts x and a fresh output at different
    # phases: the default picks the register kernel, an explicit stream config
    # is refused.
    odd = base[:, 3:1003]
    gate(ref.softmax_ref(host(odd)), softmax(odd), torch.bfloat16)
    from kernelo_b200.runtime.native import OutOfResources

    with pytest.raises(OutOfResources, match="phase"):
        softmax(odd, config=stream_cfg("softmax", 1000, num_warps=1))


def test_softmax_default_kernel_by_row_width(device):
    """Many rows: rows up to 2 KB go a warp per row (on the 16-byte grid) or
    stream (two slots per group), rows up to 64 KB sit in registers at ~8
    vectors per thread, wider rows stream; few rows, or x off the output's
    16-byte phase, stay in registers. Each default also runs and passes the
    gate."""
    from kernelo_b200.kernels.rows_common import default_rows_config

    x = rand(4096, 4096, torch.float16, device)
    narrow = rand(4096, 1000, torch.float16, device)
    cfg = default_rows_config("softmax", 1000, torch.float16, rows=4096, x=narrow)
    assert (cfg["ROW_KERNEL"], cfg["num_warps"]) == (3, 1)
    gate(ref.softmax_ref(host(narrow)), softmax(narrow), torch.float16)
    ragged = rand(4096, 1001, torch.float16, device)  # not whole vectors: streamed
    cfg = default_rows_config("softmax", 1001, torch.float16, rows=4096, x=ragged)
    assert (cfg["ROW_KERNEL"], cfg["num_warps"], cfg["num_stages"]) == (2, 1, 2)
    gate(ref.softmax_ref(host(ragged)), softmax(ragged), torch.float16)
    cfg = default_rows_config("softmax", 4096, torch.float16, rows=4096, x=x)
    assert (cfg["ROW_KERNEL"], cfg["num_warps"]) == (1, 2)
    gate(ref.softmax_ref(host(x)), softmax(x), torch.float16)
    assert default_rows_config("softmax", 8192, torch.float16, rows=4096)["num_warps"] == 4
    assert default_rows_config("softmax", 1000, torch.float16, rows=64, x=narrow[:64])["ROW_KERNEL"] == 1
    assert default_rows_config("softmax", 32000, torch.float32, rows=32768)["ROW_KERNEL"] == 2
    assert default_rows_config("rmsnorm", 4096, torch.float16, rows=16384, x=x)["ROW_KERNEL"] == 1
    assert default_rows_config("rmsnorm", 1024, torch.float16, rows=16384)["ROW_KERNEL"] == 3
    assert default_rows_config("rmsnorm", 2048, torch.float16, rows=16384)["ROW_KERNEL"] == 3
    assert default_rows_config("rmsnorm", 4096, torch.float16, rows=16384)["ROW_KERNEL"] == 1
    assert default_rows_config("softmax", 2048, torch.float16, rows=16384)["ROW_KERNEL"] == 1
    gamma = (rand(1, 1000, torch.float32, device, seed=1)[0] * 0.1 + 1).half()
    gate(ref.rmsnorm_ref(host(narrow), host(gamma), 1e-6), rmsnorm(narrow, gamma, eps=1e-6), torch.float16)


def test_stream_kernel_rejects_bad_configs(device):
    from kernelo_b200.runtime.native import OutOfResources

    x = rand(400, 4096, torch.float32, device)
    with pytest.raises(OutOfResources, match="register pressure"):
        softmax(x, config=stream_cfg("softmax", 4096, num_warps=1))  # 32 vectors per thread
    with pytest.raises(OutOfResources, match="16 warps"):
        softmax(x, config=stream_cfg("softmax", 4096, num_warps=8, ROW_GROUPS=3))
    with pytest.raises(OutOfResources, match="row slots"):
        softmax(x, config=stream_cfg("softmax", 4096, num_warps=8, num_stages=40))


# ---------------------------------------------------------------- warp-per-row kernel
def warp_cfg(op, cols):
    return KernelConfig(op, BLOCK_SIZE=max(1, 1 << (cols - 1).bit_length()), ROW_KERNEL=3, num_warps=1)


@pytest.mark.parametrize("cols", [8, 16, 64, 248, 256, 264, 512, 1000, 1024, 1536, 2048])
@pytest.mark.parametrize("dtype", DTYPES, ids=lambda d: str(d)[6:])
@pytest.mark.parametrize("rows", [1, 7, 301, 5000])
def test_warp_kernel_widths(cols, dtype, rows, device):
    """One to four vectors per lane (the three instantiations), rows fewer
    than one CTA's 8 warps, more rows than resident warps (each warp loops),
    padding lanes of a partial last vector group; both operations."""
    if cols * dtype.itemsize > 4096:
        pytest.skip("rows beyond 4 KB are not the warp kernel's")
    x = rand(rows, cols, dtype, device, scale=4.0, seed=cols)
    y = torch.full_like(x, float("nan"))
    from kernelo_b200.runtime import native

    native.softmax_rows(x, y, warp_cfg("softmax", cols))
    gate(ref.softmax_ref(host(x)), y, dtype, context=f"softmax {rows}x{cols}")
    gamma = (rand(1, cols, torch.float32, device, seed=1)[0] * 0.1 + 1).to(dtype)
    y = torch.full_like(x, float("nan"))
    native.rmsnorm_rows(x, gamma, y, 1e-6, warp_cfg("rmsnorm", cols))
    gate(ref.rmsnorm_ref(host(x), host(gamma), 1e-6), y, dtype, context=f"rmsnorm {rows}x{cols}")


def test_warp_kernel_edge_rows(device):
    """A -inf row mixed in (all but one element), a row of one value, huge
    logits; a strided view whose rows stay on the 16-byte grid."""
    x = rand(600, 1000, torch.float16, device, scale=4.0)
    x[3] = float("-inf")
    x[3, 17] = 1.0
    x[5] = 7.0
    x[9, 100] = 60000.0
    out = softmax(x, config=warp_cfg("softmax", 1000))
    assert out[3, 17].item() == 1.0 and float(out[3].float().sum()) == 1.0
    assert torch.allclose(out[5].float(), torch.full((1000,), 1e-3, device=device), rtol=1e-3)
    assert out[9, 100].item() == 1.0
    gate(ref.softmax_ref(host(x)), out, torch.float16)
    base = rand(700, 1536, torch.bfloat16, device, scale=4.0)
    view = base[:, 64:1088]  # 1024 columns, row pitch 3 KB, start on the grid
    gate(ref.softmax_ref(host(view)), softmax(view, config=warp_cfg("softmax", 1024)), torch.bfloat16)
    gamma = torch.ones(1024, device=device, dtype=torch.bfloat16)
    gate(ref.rmsnorm_ref(host(view), host(gamma)), rmsnorm(view, gamma, config=warp_cfg("rmsnorm", 1024)),
         torch.bfloat16)


def test_warp_kernel_refuses_layouts_it_cannot_take(device):
    from kernelo_b200.runtime.native import OutOfResources

    x = rand(400, 1001, torch.float16, device)
    with pytest.raises(OutOfResources, match="whole 16-byte vectors"):
        softmax(x, config=warp_cfg("softmax", 1001))
    wide = rand(400, 4096, torch.float16, device)
    with pytest.raises(OutOfResources, match="4 KB"):
        softmax(wide, config=warp_cfg("softmax", 4096))
    odd = rand(400, 1032, torch.float16, device)[:, 4:1028]  # start 8 bytes off the grid
    with pytest.raises(OutOfResources, match="16-byte grid"):
        softmax(odd, config=warp_cfg("softmax", 1024))
    # the default routes the same view elsewhere and is still right
    gate(ref.softmax_ref(host(odd)), softmax(odd), torch.float16)


@pytest.mark.parametrize("cols", [1, 7, 1000, 4096, 4097, 32000])
@pytest.mark.parametrize("kernel", [1, 2, 3])
def test_row_kernels_write_every_output(cols, kernel, device):
    """Outputs start as NaN, so a row or a tail the kernel skipped fails the
    finiteness check; both kernels, narrow to 128 KiB rows, unaligned widths."""
    from kernelo_b200.kernels.rows_common import stream_fits
    from kernelo_b200.runtime import native
    from kernelo_b200.tuning.config import KernelConfig

    dtype = torch.float32 if cols == 32000 else torch.float16
    rows = 300 if kernel == 2 else 37
    if kernel == 2 and not stream_fits(cols, dtype):
        pytest.skip("row does not fit a streaming slot")
    if kernel == 3 and (cols * dtype.itemsize % 16 or cols * dtype.itemsize > 2048):
        pytest.skip("not a warp-kernel row")
    x = rand(rows, cols, dtype, device)
    gamma = rand(1, cols, dtype, device)[0]
    block = max(1, 1 << (cols - 1).bit_length())
    cfg = KernelConfig("softmax", BLOCK_SIZE=block, ROW_KERNEL=kernel)
    y = torch.full_like(x, float("nan"))
    native.softmax_rows(x, y, cfg)
    assert torch.isfinite(y).all()
    gate(ref.softmax_ref(host(x)), y, dtype)
    y = torch.full_like(x, float("nan"))
    native.rmsnorm_rows(x, gamma, y, 1e-5, KernelConfig("rmsnorm", BLOCK_SIZE=block, ROW_KERNEL=kernel))
    assert torch.isfinite(y).all()
    gate(ref.rmsnorm_ref(host(x), host(gamma)), y, dtype)
