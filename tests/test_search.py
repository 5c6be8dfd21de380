"""sm_100a search spaces: every filter rule named and checked against the
configuration it exists to reject, on device capabilities passed in as values
(no GPU needed). The reference's rules (tuning/search.py:259-503) are
regenerated for Blackwell: tcgen05 tiles, TMEM columns, 227 KiB shared memory,
TMA alignment, swizzle atoms and thread-block clusters.
"""

from __future__ import annotations

import pytest
import torch

from kernelo_b200.kernels import gemm_common as gc
from kernelo_b200.tuning.config import KernelConfig, Problem
from kernelo_b200.tuning.search import (
    DEFAULT_MAX_CANDIDATES,
    FusedLinearErfSearchSpace,
    FusedLinearSearchSpace,
    GemvSearchSpace,
    MatmulSearchSpace,
    RMSNormSearchSpace,
    SoftmaxSearchSpace,
    next_power_of_2,
    search_space,
)

GEMM = Problem.create("matmul", "fp16", M=2048, N=4096, K=4096)
FUSED = Problem.create("fused_linear_erf", "bf16", M=4096, N=11008, K=4096)


def tc(op="matmul", **kw):
    base = dict(KERNEL=1, BLOCK_M=128, BLOCK_N=256, BLOCK_K=64, GROUP_M=8, num_stages=4, STREAM_K=2,
                SWAP_AB=2, CLUSTER_N=1)
    base.update(kw)
    base.setdefault("CLUSTER_M", 2 if base["BLOCK_M"] == 256 else 1)
    return KernelConfig(op, **base)


@pytest.mark.parametrize("n,expected", [(1, 1), (3, 4), (127, 128), (128, 128), (4097, 8192)])
def test_next_power_of_2(n, expected):
    assert next_power_of_2(n) == expected


def test_grid_size_and_budget(b200_caps):
    result = MatmulSearchSpace().generate(GEMM, b200_caps)
    # the column GEMV + tcgen05 grid (2 x 6 x 2 x 5 x 3) + SIMT tiles; the library default is one of them here
    assert result.generated == 1 + 2 * 6 * 2 * 5 * 3 + 3
    default = MatmulSearchSpace().library_default(GEMM)
    assert result.candidates[0] == default, "the library default is always measured, first"
    assert 0 < result.feasible < result.generated
    assert len(result.candidates) <= DEFAULT_MAX_CANDIDATES
    assert len(set(result.candidates)) == len(result.candidates)
    assert MatmulSearchSpace().candidates(GEMM, b200_caps) == MatmulSearchSpace().candidates(GEMM, b200_caps)
    assert len(MatmulSearchSpace().candidates(GEMM, b200_caps, max_candidates=5)) == 5


def test_flagship_shape_prefers_sm_pair_tiles(b200_caps):
    best = FusedLinearErfSearchSpace().candidates(FUSED, b200_caps)[0]
    assert best["KERNEL"] == gc.KERNEL_TCGEN05 and best["BLOCK_N"] == 256 and best["BLOCK_M"] == 256
    assert (best["CLUSTER_M"], best["CLUSTER_N"]) == (2, 1)


def test_sm_pair_tiles_are_feasible_and_sized_per_cta(b200_caps):
    space = MatmulSearchSpace()
    pair = tc(BLOCK_M=256, CLUSTER_M=2, BLOCK_N=256, num_stages=6)
    assert space.reject_reason(pair, GEMM, b200_caps) is None
    # each CTA stages 128 rows of A and half of B: 6 x (128 + 128) x 64 x 2 bytes
    assert space.shared_memory_bytes(pair, GEMM) == 6 * 256 * 64 * 2 + 1024 + 8 * 17 + 16
    assert space.num_programs(pair, GEMM) == 2 * (2048 // 256) * (4096 // 256)


@pytest.mark.parametrize(
    "config,rule",
    [
        (tc(BLOCK_N=256, BLOCK_K=64, num_stages=6), "shared memory"),
        (tc(BLOCK_K=32), "swizzle atom"),
        (tc(BLOCK_M=256, BLOCK_N=16), "SM pair"),
        (tc(BLOCK_M=256, BLOCK_N=192), "MN-major B"),
        (tc(BLOCK_N=16), "MN-major B"),  # matmul's B is row-major (K, N)
        (tc(BLOCK_N=256, num_stages=6, BLOCK_K=128), "shared memory"),
        (tc(BLOCK_M=256, BLOCK_N=128, STREAM_K=3), "split tail"),  # 64-column halves of a pair tile
    ],
)
def test_each_rule_rejects_its_config(config, rule, b200_caps):
    reason = MatmulSearchSpace().reject_reason(config, GEMM, b200_caps)
    assert reason is not None and reason.startswith(rule), reason


def test_schedule_rules(b200_caps):
    """Every point of the grid is a schedule the kernel runs: the split tail
    only where the last wave is partial, stream-K only within its counters."""
    space = FusedLinearErfSearchSpace()
    whole_waves = Problem.create("fused_linear_erf", "bf16", M=128 * 148, N=256, K=1024)  # 148 one-SM tiles
    reason = space.reject_reason(tc("fused_linear_erf", STREAM_K=3, BLOCK_N=256), whole_waves, b200_caps)
    assert reason is not None and "no partial last wave" in reason
    assert space.reject_reason(tc("fused_linear_erf", STREAM_K=2, BLOCK_N=256), whole_waves, b200_caps) is None
    huge = Problem.create("fused_linear_erf", "bf16", M=65536, N=65536, K=1024)
    reason = space.reject_reason(tc("fused_linear_erf", STREAM_K=1, BLOCK_N=128), huge, b200_caps)
    assert reason is not None and reason.startswith("stream-K")
    # no cluster shape, M=64 tile or other point the kernels cannot run is left in the grid
    for config in space.grid(FUSED):
        if config["KERNEL"] == gc.KERNEL_TCGEN05:
            assert config["BLOCK_M"] in (128, 256) and config["CLUSTER_N"] == 1
            assert config["CLUSTER_M"] == (2 if config["BLOCK_M"] == 256 else 1)
            assert config["STREAM_K"] in (1, 2, 3)


def test_tmem_budget_is_a_device_property(b200_caps, a100_caps):
    """A double-buffered 256-column accumulator fits B200's 512 TMEM columns;
    a device without TMEM rejects every tcgen05 tile."""
    space = FusedLinearErfSearchSpace()
    assert space.reject_reason(tc("fused_linear_erf"), FUSED, b200_caps) is None
    reason = space.reject_reason(tc("fused_linear_erf"), FUSED, a100_caps)
    assert reason is not None and ("TMEM" in reason or "shared memory" in reason)


def test_fp32_runs_as_3xtf32_and_unaligned_16bit_packs(b200_caps):
    """fp32 beyond 64 x 64 runs as 3xTF32 tcgen05 tiles on split operands (K is
    three 32-aligned segments, BLOCK_K one or two 32-element atoms, B K-major
    whatever its layout), the CUDA-core tiles staying candidates; 16-bit
    operands TMA cannot describe (the prime sweep shapes) are packed for
    tcgen05, which becomes the library default."""
    fp32 = Problem.create("matmul", "fp32", M=4099, N=4099, K=4099)
    space = MatmulSearchSpace()
    cands = space.candidates(fp32, b200_caps)
    assert cands[0]["KERNEL"] == gc.KERNEL_TCGEN05 and cands[0]["BLOCK_K"] in (32, 64)
    assert space.tc_k(fp32) == gc.tf32_split_k(4099) == 4128
    assert {c["BLOCK_K"] for c in cands if c["KERNEL"] == gc.KERNEL_TCGEN05} <= {32, 64}
    assert any(c["KERNEL"] == gc.KERNEL_SIMT for c in space.grid(fp32))
    # the split B is K-major: 16-column tiles are not refused as MN-major boxes
    narrow = KernelConfig("matmul", KERNEL=1, BLOCK_M=128, BLOCK_N=16, BLOCK_K=32, GROUP_M=1, num_stages=4,
                          STREAM_K=2, SWAP_AB=2, CLUSTER_M=1, CLUSTER_N=1)
    assert "MN-major" not in (space.reject_reason(narrow, fp32, b200_caps) or "")
    assert space.reject_reason(narrow.replace(BLOCK_K=16), fp32, b200_caps).startswith("swizzle atom")
    assert space.reject_reason(narrow.replace(BLOCK_K=128), fp32, b200_caps).startswith("swizzle atom")
    small = gc.default_gemm_config("matmul", 64, 4096, 4096, torch.float32, b_layout="kn")
    assert small["KERNEL"] == gc.KERNEL_SIMT, "skinny fp32 keeps IEEE FMA in place"
    for problem in (Problem.create("matmul", "fp16", M=4099, N=4099, K=4099),
                    Problem.create("matmul", "bf16", M=1021, N=2053, K=509)):
        cands = MatmulSearchSpace().candidates(problem, b200_caps)
        assert cands[0]["KERNEL"] == gc.KERNEL_TCGEN05, "packed tcgen05 is the library default"
        assert any(c["KERNEL"] == gc.KERNEL_SIMT for c in MatmulSearchSpace().grid(problem))
    skinny = Problem.create("matmul", "fp16", M=16, N=2053, K=509)  # skinny: no copy by default
    assert MatmulSearchSpace().library_default(skinny)["KERNEL"] == gc.KERNEL_SIMT
    assert gc.packs_by_default(4099, 4099, 4099, torch.float16, b_layout="kn")
    assert not gc.packs_by_default(4096, 4096, 4096, torch.float16, b_layout="kn")


@pytest.mark.parametrize("m", [1, 4, 16])
def test_decode_shapes_swap_and_keep_the_smallest_tile(m, b200_caps):
    problem = Problem.create("gemv", "fp16", M=m, N=11008, K=4096)
    cands = GemvSearchSpace().candidates(problem, b200_caps)
    tcs = [c for c in cands if c["KERNEL"] == gc.KERNEL_TCGEN05]
    assert tcs and all(c["SWAP_AB"] == 1 and c["BLOCK_N"] == 16 for c in tcs)


def test_pipeline_fill_rule(b200_caps):
    shallow = Problem.create("matmul", "fp16", M=2048, N=2048, K=128)
    reason = MatmulSearchSpace().reject_reason(tc(num_stages=4, BLOCK_N=128), shallow, b200_caps)
    assert reason is not None and reason.startswith("pipeline cannot fill")


def test_underutilisation_prune(b200_caps):
    problem = Problem.create("matmul", "fp16", M=1024, N=4096, K=1024)
    result = MatmulSearchSpace().generate(problem, b200_caps)
    space = MatmulSearchSpace()
    assert all(space.num_programs(c, problem) >= b200_caps.sm_count // 2 for c in result.candidates)
    tiny = Problem.create("matmul", "fp16", M=64, N=64, K=256)
    r = space.generate(tiny, b200_caps)
    assert r.after_prune == r.feasible and r.candidates


def test_explain_names_rules_and_device(b200_caps):
    text = MatmulSearchSpace().explain(GEMM, b200_caps)
    assert "NVIDIA B200" in text and "grid points" in text and "rejections by rule" in text


def test_row_space_shape_and_rules(b200_caps):
    problem = Problem.create("rmsnorm", "fp16", rows=16384, cols=4096)
    cands = RMSNormSearchSpace().candidates(problem, b200_caps, max_candidates=1000)
    register = [c for c in cands if c["ROW_KERNEL"] == 1]
    stream = [c for c in cands if c["ROW_KERNEL"] == 2]
    assert register and {k for c in register for k in c} == {
        "ROW_KERNEL", "BLOCK_SIZE", "ROWS_PER_PROGRAM", "num_warps", "CLUSTER"}
    assert stream and {k for c in stream for k in c} == {"ROW_KERNEL", "BLOCK_SIZE", "num_warps", "num_stages"}
    assert sorted({c["num_warps"] for c in stream}) == [1, 2, 4, 8, 16]
    assert cands[0]["ROW_KERNEL"] == 1, "RMSNorm: the register kernel (library default) ranks first"
    # softmax: 8 KB rows in registers at ~8 vectors per thread (2 warps), 2 KB
    # rows a warp per row, then the streaming kernel
    soft = Problem.create("softmax", "fp16", rows=16384, cols=4096)
    first = SoftmaxSearchSpace().candidates(soft, b200_caps)[0]
    assert (first["ROW_KERNEL"], first["num_warps"], first["CLUSTER"]) == (1, 2, 1)
    soft_narrow = Problem.create("softmax", "fp16", rows=32768, cols=1000)
    narrow_cands = SoftmaxSearchSpace().candidates(soft_narrow, b200_caps)
    assert (narrow_cands[0]["ROW_KERNEL"], narrow_cands[0]["num_warps"]) == (3, 1)
    assert any(c["ROW_KERNEL"] == 2 for c in narrow_cands)
    # 8 KB rows exceed the warp kernel; odd rows of fp16 do not hold whole vectors
    warp = KernelConfig("softmax", BLOCK_SIZE=4096, ROW_KERNEL=3, num_warps=1)
    assert "exceeds 4 KB" in SoftmaxSearchSpace().reject_reason(warp, soft, b200_caps)
    odd = Problem.create("softmax", "fp16", rows=32768, cols=999)
    assert "whole 16-byte vectors" in SoftmaxSearchSpace().reject_reason(warp.replace(BLOCK_SIZE=1024), odd,
                                                                          b200_caps)
    assert SoftmaxSearchSpace().candidates(odd, b200_caps)[0]["ROW_KERNEL"] == 2
    assert {c["BLOCK_SIZE"] for c in cands} == {4096}
    wide = Problem.create("softmax", "fp32", rows=32768, cols=32000)
    space = SoftmaxSearchSpace()
    one_cta = KernelConfig("softmax", BLOCK_SIZE=32768, ROWS_PER_PROGRAM=1, num_warps=4, CLUSTER=1)
    assert space.reject_reason(one_cta, wide, b200_caps).startswith("register pressure")
    assert any(c.get("CLUSTER", 1) > 1 for c in space.candidates(wide, b200_caps))
    # 8000 vectors: 16 streaming warps hold 16 each; 8 would need 32
    st16 = KernelConfig("softmax", BLOCK_SIZE=32768, ROW_KERNEL=2, num_warps=16)
    st8 = KernelConfig("softmax", BLOCK_SIZE=32768, ROW_KERNEL=2, num_warps=8)
    assert space.reject_reason(st16, wide, b200_caps) is None
    assert space.reject_reason(st8, wide, b200_caps).startswith("register pressure")
    few = Problem.create("softmax", "fp16", rows=64, cols=4096)
    st4 = KernelConfig("softmax", BLOCK_SIZE=4096, ROW_KERNEL=2, num_warps=4)
    assert "rows leave persistent CTAs" in space.reject_reason(st4, few, b200_caps)
    assert space.candidates(few, b200_caps)[0]["ROW_KERNEL"] == 1
    narrow = Problem.create("softmax", "fp16", rows=32768, cols=1000)  # 125 vectors
    st8 = KernelConfig("softmax", BLOCK_SIZE=1024, ROW_KERNEL=2, num_warps=8)
    assert space.reject_reason(st8, narrow, b200_caps).startswith("idle threads")
    huge = Problem.create("softmax", "fp32", rows=4096, cols=65536)  # 256 KiB rows
    st = KernelConfig("softmax", BLOCK_SIZE=65536, ROW_KERNEL=2, num_warps=16)
    assert "shared-memory slot" in space.reject_reason(st, huge, b200_caps)
    too_wide = Problem.create("softmax", "fp16", rows=2, cols=300_000)
    assert all(r.startswith("row of") for _, r in space.generate(too_wide, b200_caps).rejected)


def test_default_configs_are_feasible(b200_caps):
    from kernelo_b200.kernels import get_operator

    for op_name, problem in (
        ("matmul", GEMM),
        ("fused_linear_erf", FUSED),
        ("gemv", Problem.create("gemv", "fp16", M=1, N=11008, K=4096)),
        ("softmax", Problem.create("softmax", "fp32", rows=32768, cols=32000)),
        ("rmsnorm", Problem.create("rmsnorm", "bf16", rows=16384, cols=8192)),
    ):
        op = get_operator(op_name)
        cfg = op.default_config(problem)
        assert op.search_space().reject_reason(cfg, problem, b200_caps) is None, (op_name, cfg)


def test_unknown_space_is_an_error():
    with pytest.raises(ValueError):
        search_space("vector_add")
    assert isinstance(search_space("gemv"), GemvSearchSpace)


def test_gemv_tile_rows_candidates(b200_caps):
    """The 16-row tile kernel leads for 16-bit x up to 16 rows, its default
    shape first; fp32, M > 16 and K % 8 != 0 reject it."""
    space = GemvSearchSpace()
    for m, default in ((1, (8, 1)), (4, (8, 1)), (16, (6, 4))):
        p = Problem.create("gemv", "bf16", M=m, N=11008, K=4096)
        cands = space.candidates(p, b200_caps)
        assert cands[0]["KERNEL"] == gc.KERNEL_TILE_ROWS
        assert (cands[0]["BLOCK_M"], cands[0]["num_stages"]) == default
        tiles = [c for c in cands if c["KERNEL"] == gc.KERNEL_TILE_ROWS]
        assert len(tiles) == len(gc.TILE_ROWS_SHAPES)
        assert space.num_programs(tiles[0], p) == 688
    tile = KernelConfig("gemv", KERNEL=gc.KERNEL_TILE_ROWS, BLOCK_M=8, num_stages=2)
    assert space.reject_reason(tile, Problem.create("gemv", "fp32", M=1, N=64, K=64), b200_caps).startswith(
        "the tile GEMV takes fp16 or bf16")
    assert "1..32 rows" in space.reject_reason(tile, Problem.create("gemv", "fp16", M=33, N=64, K=64), b200_caps)
    assert "K % 8" in space.reject_reason(tile, Problem.create("gemv", "fp16", M=2, N=64, K=4099), b200_caps)


def test_fused_linear_decode_shapes_take_tile_rows(b200_caps):
    from kernelo_b200.tuning.search import FusedLinearErfSearchSpace, MatmulSearchSpace

    for m, expected in ((1, 4), (16, 4), (32, 4), (33, 1), (4096, 1)):
        cfg = gc.default_gemm_config("fused_linear_erf", m, 11008, 4096, torch.bfloat16, b_layout="nk")
        assert cfg["KERNEL"] == expected, (m, cfg)
    decode = Problem.create("fused_linear_erf", "bf16", M=4, N=11008, K=4096)
    first = FusedLinearErfSearchSpace().candidates(decode, b200_caps)[0]
    assert (first["KERNEL"], first["BLOCK_M"], first["num_stages"]) == (4, 8, 1)
    # a row-major (K, N) B is not K-contiguous: no tile candidates for matmul
    mm = Problem.create("matmul", "fp16", M=4, N=4096, K=4096)
    assert all(c["KERNEL"] != 4 for c in MatmulSearchSpace().candidates(mm, b200_caps))
    # (up to 8 rows against a row-major B take the column GEMV; 16 rows take swapped tcgen05 tiles)
    assert gc.default_gemm_config("matmul", 4, 4096, 4096, torch.float16, b_layout="kn")["KERNEL"] == 5
    assert gc.default_gemm_config("matmul", 16, 4096, 4096, torch.float16, b_layout="kn")["KERNEL"] == 1


def test_row_major_b_decode_shapes_take_the_column_gemv(b200_caps):
    """M <= 8 against a row-major (K, N) B: the column GEMV, any dtype, leads;
    wider M, N off the 16-byte grid or an [N, K] weight reject it."""
    for dtype in ("fp16", "bf16", "fp32"):
        p = Problem.create("matmul", dtype, M=1, N=11008, K=4096)
        first = MatmulSearchSpace().candidates(p, b200_caps)[0]
        assert first["KERNEL"] == gc.KERNEL_COLUMNS, (dtype, first)
        assert MatmulSearchSpace().num_programs(first, p) >= b200_caps.sm_count
    cols = KernelConfig("matmul", KERNEL=gc.KERNEL_COLUMNS)
    space = MatmulSearchSpace()
    assert "1..8 rows" in space.reject_reason(cols, Problem.create("matmul", "fp16", M=16, N=4096, K=64), b200_caps)
    assert "multiple of 8" in space.reject_reason(cols, Problem.create("matmul", "fp16", M=2, N=2053, K=64),
                                                  b200_caps)
    assert "N-contiguous" in FusedLinearSearchSpace().reject_reason(
        KernelConfig("fused_linear", KERNEL=gc.KERNEL_COLUMNS), Problem.create("fused_linear", "fp16", M=1, N=64,
                                                                               K=64), b200_caps)


def test_gemv_warp_rows_candidate(b200_caps):
    space = GemvSearchSpace()
    # fp32 x: the tile kernel is out, the warp-per-row kernel is the default at M <= 2
    one = Problem.create("gemv", "fp32", M=1, N=11008, K=4096)
    cands = space.candidates(one, b200_caps)
    assert cands[0]["KERNEL"] == gc.KERNEL_WARP_ROWS, "M=1 fp32: the warp-per-row kernel is the default"
    four = Problem.create("gemv", "fp16", M=4, N=11008, K=4096)
    cands4 = space.candidates(four, b200_caps)
    assert any(c["KERNEL"] == 3 for c in cands4)
    wide = Problem.create("gemv", "fp16", M=16, N=11008, K=4096)
    warp_rows = KernelConfig("gemv", KERNEL=gc.KERNEL_WARP_ROWS)
    assert space.reject_reason(warp_rows, wide, b200_caps).startswith("warp-per-row GEMV takes at most 4")
    # x staged as fp32: 4 rows x 16384 columns = 256 KiB of shared memory
    long_k = Problem.create("gemv", "fp16", M=4, N=1024, K=16384)
    assert space.reject_reason(warp_rows, long_k, b200_caps).startswith("shared memory")
    assert gc.warp_rows_smem_bytes(1, 4096, 2) == 1 * (4096 + 8) * 4
