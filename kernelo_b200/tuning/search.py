"""Candidate generation for sm_100a.

The reference's tuner takes its candidates from a hardware-derived grid,
rejects points with a named reason, drops launches that would leave most SMs
idle, and budgets the rest by a documented priority
(``kernelforge/tuning/search.py:122-217``). That contract is kept; the grids
and rules are Blackwell's, and every grid point is a configuration this
library's kernels can actually run:

GEMM (``matmul``, ``fused_linear``, ``fused_linear_erf``, ``gemv``)
    tcgen05 tiles: ``BLOCK_M`` {128 (one SM), 256 (an SM pair, cta_group::2,
    on a 2x1 cluster)} x ``BLOCK_N`` {16, 64, 128, 192, 224, 256} x
    ``BLOCK_K`` {one, two 128-byte swizzle atoms: 64, 128 16-bit or 32, 64
    fp32 elements} x ``num_stages`` (shared-memory ring depth)
    {2, 3, 4, 6, 8} x ``STREAM_K`` (tile schedule: 1 stream-K, 2 whole
    tiles, 3 whole tiles with the last partial wave split into half-width
    tiles) = 360 points; ``SWAP_AB`` follows the shape (skinny M puts the
    weight on the 128-row side) and ``GROUP_M`` (the L2 raster width) the
    library's rule. fp32 tiles run as 3xTF32 on split K-major operands (the
    kernel's K is three TF32 segments). Plus the 16-row tile GEMV's compiled
    shapes for K-contiguous weights, the column GEMV for an N-contiguous B,
    and the CUDA-core tiles (IEEE fp32, any strides).

    Limits applied as named rules: 227 KiB of shared memory per CTA, 512
    TMEM columns per SM (a double-buffered fp32 accumulator takes 2 x
    BLOCK_N), TMA's 16-byte stride rule, an MN-major B in 64-column boxes, a
    pair tile's BLOCK_N split in two 16-column-aligned halves, tile overshoot,
    pipeline fill, and the schedules' own conditions.

Row reductions (``softmax``, ``rmsnorm``)
    The register kernel: ``num_warps`` {1..32} x ``ROWS_PER_PROGRAM``
    {1, 2, 4} x ``CLUSTER`` {1, 2, 4, 8} (CTAs sharing one row through
    distributed shared memory); the streaming kernel: warps per row group
    {1..16} with as many or with two shared-memory slots per group.
    ``BLOCK_SIZE`` (next power of two of the row) is kept for the reference's
    "cannot hold a row" / "single-pass limit" checks; the single-pass limit
    is 131072 columns because a row may span a cluster.

Filters read a :class:`DeviceCaps` value, never ``torch.cuda``, so they can be
tested against a GPU that is not attached. A :class:`CandidateSet` records
how many configs survived each stage of the funnel.
"""

from __future__ import annotations

import math
import re
from abc import ABC, abstractmethod
from collections import Counter
from collections.abc import Iterator
from dataclasses import dataclass
from itertools import product

import torch

from kernelo_b200.dtypes import itemsize
from kernelo_b200.kernels import gemm_common as gc
from kernelo_b200.runtime.env import DeviceCaps, device_caps
from kernelo_b200.tuning.config import KernelConfig, Problem

DEFAULT_MAX_CANDIDATES = 48


def next_power_of_2(n: int) -> int:
    if n < 1:
        raise ValueError(f"expected a positive integer, got {n}")
    return 1 << (n - 1).bit_length()


def ceil_div(a: int, b: int) -> int:
    return -(-a // b)


@dataclass(frozen=True)
class CandidateSet:
    """The funnel's result: the budgeted candidates, what each stage left, and
    every rejected config with its reason."""

    problem: Problem
    generated: int
    feasible: int
    after_prune: int
    budget: int
    candidates: list[KernelConfig]
    rejected: tuple[tuple[KernelConfig, str], ...]

    def __len__(self) -> int:
        return len(self.candidates)

    def __iter__(self) -> Iterator[KernelConfig]:
        return iter(self.candidates)

    def rule_counts(self) -> Counter:
        """Rejections per rule: a reason's text before its first ':' or '('."""
        return Counter(re.split(r"[:(]", reason, maxsplit=1)[0].strip() for _, reason in self.rejected)


class SearchSpace(ABC):
    """Configurations worth trying for one operation.

    Subclasses give the grid, the rejection rules and (optionally) the launch
    size and the budget priority; :meth:`generate` runs the funnel."""

    operation: str

    def __init__(self, max_candidates: int = DEFAULT_MAX_CANDIDATES) -> None:
        if max_candidates < 1:
            raise ValueError(f"max_candidates must be positive, got {max_candidates}")
        self.max_candidates = max_candidates

    @abstractmethod
    def grid(self, problem: Problem) -> Iterator[KernelConfig]: ...

    @abstractmethod
    def reject_reason(self, config: KernelConfig, problem: Problem, caps: DeviceCaps) -> str | None:
        """Why ``config`` is not worth trying, or None to keep it."""

    def num_programs(self, config: KernelConfig, problem: Problem) -> int:
        """CTAs the launch would have; spaces that cannot say raise."""
        raise NotImplementedError

    def priority(self, config: KernelConfig, problem: Problem, caps: DeviceCaps) -> tuple[float, ...]:
        """Budget sort key, lower first (ties broken by the serialised config)."""
        return (0.0,)

    def candidates(
        self, problem: Problem, caps: DeviceCaps | None = None, *, max_candidates: int | None = None
    ) -> list[KernelConfig]:
        return self.generate(problem, caps, max_candidates=max_candidates).candidates

    # ------------------------------------------------------------ the funnel
    def _feasibility(self, problem: Problem, caps: DeviceCaps):
        """Stage 1: every grid point, kept or rejected with its rule."""
        kept, rejected, seen = [], [], 0
        for config in self.grid(problem):
            seen += 1
            reason = self.reject_reason(config, problem, caps)
            if reason is None:
                kept.append(config)
            else:
                rejected.append((config, reason))
        return seen, kept, rejected

    def _occupancy(self, configs: list[KernelConfig], problem: Problem, caps: DeviceCaps):
        """Stage 2: launches that fill under half the SMs go, unless no
        feasible config fills them all (then nothing is dropped)."""
        try:
            sizes = [self.num_programs(c, problem) for c in configs]
        except NotImplementedError:
            return configs, []
        if not sizes or max(sizes) < caps.sm_count:
            return configs, []
        floor = caps.sm_count // 2
        keep = [c for c, n in zip(configs, sizes) if n >= floor or self.protected(c, problem)]
        drop = [(c, f"launch grid of {n} programs fills under half of {caps.sm_count} SMs")
                for c, n in zip(configs, sizes) if n < floor and not self.protected(c, problem)]
        return keep, drop

    def protected(self, config: KernelConfig, problem: Problem) -> bool:
        """Configs the funnel never prunes (the GEMM spaces: the library default)."""
        return False

    def generate(
        self, problem: Problem, caps: DeviceCaps | None = None, *, max_candidates: int | None = None
    ) -> CandidateSet:
        if problem.operation != self.operation:
            raise ValueError(f"{type(self).__name__} handles {self.operation!r}, got {problem.operation!r}")
        caps = caps or device_caps()
        budget = self.max_candidates if max_candidates is None else max_candidates
        generated, feasible, rejected = self._feasibility(problem, caps)
        survivors, pruned = self._occupancy(feasible, problem, caps)
        ranked = sorted(survivors, key=lambda c: (*self.priority(c, problem, caps), c.to_json()))
        return CandidateSet(problem, generated, len(feasible), len(survivors), budget, ranked[:budget],
                            tuple(rejected + pruned))

    def explain(self, problem: Problem, caps: DeviceCaps | None = None) -> str:
        caps = caps or device_caps()
        funnel = self.generate(problem, caps)
        note = "" if caps.measured else "  <- no device attached"
        report = [
            problem.describe(),
            f"  device           : {caps.name}, {caps.sm_count} SMs, "
            f"{caps.max_shared_memory_per_block // 1024} KiB shared/block{note}",
            f"  grid points      : {funnel.generated}",
            f"  feasible         : {funnel.feasible}",
            f"  after prune      : {funnel.after_prune}",
            f"  selected (budget): {len(funnel.candidates)} of {funnel.budget}",
        ]
        rules = funnel.rule_counts()
        if rules:
            report.append("  rejections by rule:")
            report += [f"    {count:>4}  {rule}" for rule, count in rules.most_common()]
        return "\n".join(report)


# ------------------------------------------------------------------------ GEMM
class _Sm100GemmSpace(SearchSpace):
    """tcgen05 tile grid plus the SIMT fallback tiles, shared by the GEMM operators."""

    BLOCK_M = (128, 256)
    BLOCK_N = (16, 64, 128, 192, 224, 256)
    BLOCK_K = (64, 128)
    NUM_STAGES = (2, 3, 4, 6, 8)
    #: Tile schedules of the persistent kernel: 1 stream-K (the flattened
    #: (tile, k-block) space split evenly over the SMs), 2 whole tiles,
    #: 3 whole tiles with the last partial wave split into half-width tiles.
    SCHEDULES = (1, 2, 3)
    #: L2 the A panels of one raster group may take (the library default's rule).
    GROUP_L2_BYTES = 48 << 20
    #: Most output tiles stream-K keeps arrival counters for (gemm_tcgen05.cu).
    STREAM_K_MAX_TILES = 16384
    #: (BLOCK_M, BLOCK_N, BLOCK_K) of the CUDA-core kernel's instantiations.
    SIMT_TILES = ((128, 128, 8), (64, 64, 16), (128, 64, 16))
    #: How B is laid out for this operator's canonical inputs.
    b_layout = "nk"

    def dims(self, problem: Problem) -> tuple[int, int, int]:
        d = problem.dims_dict
        return d["M"], d["N"], d["K"]

    @staticmethod
    def tf32(problem: Problem) -> bool:
        """fp32 tcgen05 tiles run on TF32-split operands (3xTF32)."""
        return problem.dtype == torch.float32

    def tc_k(self, problem: Problem) -> int:
        """K as the tcgen05 kernel sees it: fp32's three TF32 segments."""
        k = self.dims(problem)[2]
        return gc.tf32_split_k(k) if self.tf32(problem) else k

    def tc_b_layout(self, problem: Problem) -> str:
        """B's layout as the tcgen05 kernel sees it: the split fp32 B is K-major."""
        return "nk" if self.tf32(problem) else self.b_layout

    def block_k_values(self, problem: Problem) -> tuple[int, ...]:
        """One or two 128-byte swizzle atoms of K."""
        atom = 128 // problem.itemsize
        return (atom, 2 * atom)

    def group_m(self, block_m: int, problem: Problem) -> int:
        """Raster group width: as many M tiles as keep their A panels within
        GROUP_L2_BYTES of L2 (so each group streams B once)."""
        m, n, _ = self.dims(problem)
        k = self.tc_k(problem)
        m_k = n if gc.default_swap(m, n) else m
        rows = max(block_m, gc.TC_BLOCK_M)
        panel = rows * k * problem.itemsize * (2 if self.tf32(problem) else 1)  # TF32: both split parts
        return max(1, min(ceil_div(m_k, rows), self.GROUP_L2_BYTES // max(1, panel)))

    def library_default(self, problem: Problem) -> KernelConfig:
        """The config the library picks on its own: always a candidate, so that
        tuning never ends worse than not tuning."""
        m, n, k = self.dims(problem)
        return gc.default_gemm_config(self.operation, m, n, k, problem.dtype, b_layout=self.b_layout)

    def protected(self, config: KernelConfig, problem: Problem) -> bool:
        return config == self.library_default(problem)

    def grid(self, problem: Problem) -> Iterator[KernelConfig]:
        default = self.library_default(problem)
        yield default
        yield from (config for config in self._grid(problem) if config != default)

    def _grid(self, problem: Problem) -> Iterator[KernelConfig]:
        m, n, _ = self.dims(problem)
        if self.b_layout == "nk":
            # decode shapes: 16-row weight tiles on mma.sync (BLOCK_M warps per
            # tile, num_stages vector pairs in flight)
            for warps, pairs in gc.TILE_ROWS_SHAPES:
                yield KernelConfig(self.operation, KERNEL=gc.KERNEL_TILE_ROWS, BLOCK_M=warps, num_stages=pairs)
            # the same tiles with the weight streamed through a shared-memory
            # ring (BLOCK_K weight elements per row per stage)
            if m <= gc.TILE_STREAM_MAX_M:
                for chunk in gc.TILE_STREAM_CHUNKS:
                    yield KernelConfig(self.operation, KERNEL=gc.KERNEL_TILE_STREAM, BLOCK_K=chunk)
        else:
            # decode shapes against a row-major (K, N) B: the column GEMV
            yield KernelConfig(self.operation, KERNEL=gc.KERNEL_COLUMNS)
        swap = 1 if gc.default_swap(m, n) else 2
        for bm, bn, bk, stages, schedule in product(self.BLOCK_M, self.BLOCK_N, self.block_k_values(problem),
                                                    self.NUM_STAGES, self.SCHEDULES):
            yield KernelConfig(self.operation, KERNEL=gc.KERNEL_TCGEN05, BLOCK_M=bm, BLOCK_N=bn, BLOCK_K=bk,
                               GROUP_M=self.group_m(bm, problem), num_stages=stages, STREAM_K=schedule,
                               SWAP_AB=swap, CLUSTER_M=gc.cta_group(bm), CLUSTER_N=1)
        for bm, bn, bk in self.SIMT_TILES:
            yield KernelConfig(self.operation, KERNEL=gc.KERNEL_SIMT, BLOCK_M=bm, BLOCK_N=bn, BLOCK_K=bk)

    def kernel_view(self, config: KernelConfig, problem: Problem) -> tuple[int, int]:
        """(M', N') the kernel tiles, after an A/B swap."""
        m, n, _ = self.dims(problem)
        return (n, m) if config.get("SWAP_AB", 2) == 1 else (m, n)

    def shared_memory_bytes(self, config: KernelConfig, problem: Problem) -> int:
        if config["KERNEL"] == gc.KERNEL_COLUMNS:
            return 0  # a few KB of reduction buffer and x slice
        if config["KERNEL"] == gc.KERNEL_TILE_STREAM:
            return gc.tile_stream_smem_bytes(self.dims(problem)[0], config["BLOCK_K"])
        if config["KERNEL"] == gc.KERNEL_TILE_ROWS:
            m = self.dims(problem)[0]
            return (config["BLOCK_M"] - 1) * 32 * gc.tile_rows_groups(m) * 16  # the K-slice partials
        if config["KERNEL"] == gc.KERNEL_SIMT:
            return 2 * config["BLOCK_K"] * (config["BLOCK_M"] + config["BLOCK_N"]) * 4
        return gc.tc_smem_bytes(config["BLOCK_N"], config["BLOCK_K"], config["num_stages"],
                                itemsize(problem.dtype), gc.cta_group(config["BLOCK_M"]))

    def output_tiles(self, config: KernelConfig, problem: Problem) -> int:
        m_k, n_k = self.kernel_view(config, problem)
        return ceil_div(m_k, config["BLOCK_M"]) * ceil_div(n_k, config["BLOCK_N"])

    def num_programs(self, config: KernelConfig, problem: Problem) -> int:
        """CTAs with work: tiles, times two for SM-pair tiles."""
        if config["KERNEL"] == gc.KERNEL_TILE_STREAM:
            # one persistent CTA per SM, never more than the 16-row tiles
            return min(gc.SM100_SMS, ceil_div(self.dims(problem)[1], 16))
        if config["KERNEL"] == gc.KERNEL_TILE_ROWS:
            # a cluster of CTAs per 16 weight rows (CLUSTER_M, else the library's split)
            m, n, _ = self.dims(problem)
            return ceil_div(n, 16) * (config.get("CLUSTER_M", 0) or gc.tile_rows_split(n, m))
        if config["KERNEL"] == gc.KERNEL_COLUMNS:
            _, n, k = self.dims(problem)
            return gc.columns_programs(n, k, problem.dtype)
        tiles = self.output_tiles(config, problem)
        if config["KERNEL"] == gc.KERNEL_TCGEN05 and config.get("STREAM_K") == 1:
            # stream-K deals the (tile, k-block) iterations over a persistent grid
            iters = tiles * ceil_div(self.tc_k(problem), config["BLOCK_K"]) * gc.cta_group(config["BLOCK_M"])
            return min(gc.SM100_SMS, iters)
        return tiles * (gc.cta_group(config["BLOCK_M"]) if config["KERNEL"] == gc.KERNEL_TCGEN05 else 1)

    def _schedule_reason(self, config: KernelConfig, problem: Problem, caps: DeviceCaps) -> str | None:
        """The tile schedules' own conditions."""
        cg = gc.cta_group(config["BLOCK_M"])
        tiles = self.output_tiles(config, problem)
        schedule = config["STREAM_K"]
        if schedule == 1 and tiles * cg > self.STREAM_K_MAX_TILES:
            return f"stream-K: {tiles} tiles exceed the {self.STREAM_K_MAX_TILES // cg} it keeps counters for"
        if schedule == 3:
            bn = config["BLOCK_N"]
            mn_major_b = self.tc_b_layout(problem) == "kn" and config["SWAP_AB"] != 1
            if (bn // 2) % (16 * cg) != 0 or (mn_major_b and (bn // cg // 2) % 64 != 0):
                return f"split tail: half of BLOCK_N={bn} is not a tile the MMA and TMA boxes take"
            units = caps.sm_count // cg
            if tiles % units == 0 or tiles < units:
                return f"split tail: {tiles} tiles leave no partial last wave on {units} units"
        return None

    def reject_reason(self, config: KernelConfig, problem: Problem, caps: DeviceCaps) -> str | None:
        m, n, k = self.dims(problem)
        if config == self.library_default(problem) and caps.is_blackwell_datacenter:
            return None  # what the library runs anyway is always measured
        if config["KERNEL"] == gc.KERNEL_TILE_ROWS:
            return gc.tile_rows_reject(m, k, problem.dtype)
        if config["KERNEL"] == gc.KERNEL_TILE_STREAM:
            return gc.tile_stream_reject(m, k, problem.dtype)
        if config["KERNEL"] == gc.KERNEL_COLUMNS:
            return gc.columns_reject(m, n, k, problem.dtype, b_layout=self.b_layout)
        if config["KERNEL"] == gc.KERNEL_SIMT:
            return None  # the fallback always runs
        why = gc.shape_allows_tcgen05(m, n, k, problem.dtype, b_layout=self.b_layout)
        if why is not None:
            return why
        bm, bn, bk, stages = config["BLOCK_M"], config["BLOCK_N"], config["BLOCK_K"], config["num_stages"]
        cg = gc.cta_group(bm)
        if bn % (16 * cg) != 0:
            return f"SM pair: BLOCK_N={bn} does not split into two 16-column halves"
        if bk * itemsize(problem.dtype) < 128:
            return f"swizzle atom: BLOCK_K={bk} is less than one 128-byte swizzle row"
        if bk * itemsize(problem.dtype) > 256:
            return f"swizzle atom: BLOCK_K={bk} is more than two 128-byte swizzle rows"
        if self.tf32(problem) and bn > 128:
            return f"TF32 register sums: BLOCK_N={bn} exceeds 128"
        smem = self.shared_memory_bytes(config, problem)
        if smem > caps.max_shared_memory_per_block:
            return (f"shared memory: {smem // 1024} KiB of tiles exceeds the "
                    f"{caps.max_shared_memory_per_block // 1024} KiB per-block limit")
        tmem = gc.tc_tmem_columns(bn)
        if tmem > caps.tmem_columns_per_sm:
            return f"TMEM: {tmem} accumulator columns exceed {caps.tmem_columns_per_sm} per SM"
        swapped = config["SWAP_AB"] == 1
        b_layout = self.tc_b_layout(problem)
        if b_layout == "kn" and not swapped and (bn // cg) % 64 != 0:
            return f"MN-major B: BLOCK_N={bn} gives each CTA a share that is not 64-column TMA boxes"
        m_k, n_k = self.kernel_view(config, problem)
        smallest = min(v for v in self.BLOCK_N if b_layout != "kn" or swapped or v % 64 == 0)
        if bn > 2 * n_k and bn > smallest:
            return f"tile overshoot: BLOCK_N={bn} for N={n_k}"
        if cg == 2 and m_k <= gc.TC_BLOCK_M:
            return f"tile overshoot: BLOCK_M={bm} for M={m_k}"
        k_iters = ceil_div(self.tc_k(problem), bk)
        if stages > 2 and k_iters < stages:
            return f"pipeline cannot fill: {k_iters} K iterations for num_stages={stages}"
        return self._schedule_reason(config, problem, caps)

    def priority(self, config: KernelConfig, problem: Problem, caps: DeviceCaps) -> tuple[float, ...]:
        """The library default first; the tile GEMV next where it runs (its
        default shape first); then tcgen05 before SIMT; then parallelism up to
        one wave; then operand reuse BM*BN/(BM+BN) (operand bytes per MMA);
        then least padding; then the schedule the library would pick for that
        tile before the other two; then the deeper ring."""
        if config == self.library_default(problem):
            return (-10,)
        if config["KERNEL"] == gc.KERNEL_TILE_ROWS:
            default = (config["BLOCK_M"], config["num_stages"]) == gc.tile_rows_default(self.dims(problem)[0])
            return (-3,) if default else (-2,)
        if config["KERNEL"] in (gc.KERNEL_COLUMNS, gc.KERNEL_TILE_STREAM):
            return (-3,)
        if config["KERNEL"] != gc.KERNEL_TCGEN05:
            return (1,)
        m_k, n_k = self.kernel_view(config, problem)
        bm, bn = config["BLOCK_M"], config["BLOCK_N"]
        programs = min(self.num_programs(config, problem), caps.sm_count)
        reuse = bm * bn / (bm + bn)
        waste = ceil_div(m_k, bm) * bm * ceil_div(n_k, bn) * bn / (m_k * n_k)
        cg = gc.cta_group(bm)
        tiles = self.output_tiles(config, problem)
        natural = 1 if (cg == 1 and tiles < caps.sm_count) else 3
        return (0, -programs, -reuse, waste, 0 if config["STREAM_K"] == natural else 1, -config["num_stages"])


class MatmulSearchSpace(_Sm100GemmSpace):
    operation = "matmul"
    b_layout = "kn"


class FusedLinearSearchSpace(_Sm100GemmSpace):
    operation = "fused_linear"
    b_layout = "nk"


class FusedLinearErfSearchSpace(_Sm100GemmSpace):
    operation = "fused_linear_erf"
    b_layout = "nk"


class GemvSearchSpace(_Sm100GemmSpace):
    """The GEMM grid plus the decode kernels: 16-row weight tiles on mma.sync
    (``KERNEL=4``; BLOCK_M warps per tile, num_stages vector pairs in flight)
    and the warp-per-row CUDA-core GEMV (``KERNEL=3``)."""

    operation = "gemv"
    b_layout = "nk"

    def library_default(self, problem: Problem) -> KernelConfig:
        from kernelo_b200.kernels.gemv import default_config

        m, n, k = self.dims(problem)
        return default_config(m, n, k, problem.dtype)

    def _grid(self, problem: Problem) -> Iterator[KernelConfig]:
        yield KernelConfig(self.operation, KERNEL=gc.KERNEL_WARP_ROWS)
        yield from super()._grid(problem)

    def shared_memory_bytes(self, config: KernelConfig, problem: Problem) -> int:
        if config["KERNEL"] == gc.KERNEL_WARP_ROWS:
            m, _, k = self.dims(problem)
            return gc.warp_rows_smem_bytes(m, k, itemsize(problem.dtype))
        return super().shared_memory_bytes(config, problem)

    def num_programs(self, config: KernelConfig, problem: Problem) -> int:
        if config["KERNEL"] == gc.KERNEL_WARP_ROWS:
            return ceil_div(self.dims(problem)[1], 16)  # 16 warps per CTA, a row or two each
        return super().num_programs(config, problem)

    def reject_reason(self, config: KernelConfig, problem: Problem, caps: DeviceCaps) -> str | None:
        if config["KERNEL"] != gc.KERNEL_WARP_ROWS:
            return super().reject_reason(config, problem, caps)
        m, _, _ = self.dims(problem)
        if m > gc.WARP_ROWS_MAX_M:
            return f"warp-per-row GEMV takes at most {gc.WARP_ROWS_MAX_M} rows of x, got M={m}"
        smem = self.shared_memory_bytes(config, problem)
        if smem > caps.max_shared_memory_per_block:
            return f"shared memory: x as fp32 needs {smem // 1024} KiB"
        return None

    def priority(self, config: KernelConfig, problem: Problem, caps: DeviceCaps) -> tuple[float, ...]:
        """The tile kernel's shapes as for every K-contiguous GEMM, then the
        warp-per-row kernel (first where it is the library default, M <= 2, and
        the tile kernel cannot run)."""
        if config["KERNEL"] == gc.KERNEL_WARP_ROWS and config != self.library_default(problem):
            return (-1,) if self.dims(problem)[0] <= gc.WARP_ROWS_AUTO_MAX_M else (2,)
        return super().priority(config, problem, caps)


# ------------------------------------------------------------------------ rows
class _RowReductionSpace(SearchSpace):
    """Row kernels. The register kernel (``ROW_KERNEL=1``): threads per CTA, rows
    per CTA, CTAs per row. The persistent streaming kernel (``ROW_KERNEL=2``):
    warps per row group, one CTA per SM with 16 consumer warps. The
    warp-per-row kernel (``ROW_KERNEL=3``): no fields, rows up to 4 KB."""

    NUM_WARPS = (1, 2, 4, 8, 16, 32)
    ROWS_PER_PROGRAM = (1, 2, 4)
    CLUSTER = (1, 2, 4, 8)
    STREAM_WARPS = (1, 2, 4, 8, 16)
    STREAM_CONSUMER_WARPS = 16
    #: Shared memory the streaming kernel keeps besides its row slots.
    STREAM_FIXED_SMEM = 128 + 8 * 16 * 16 + 16
    #: 16-byte vectors one thread may hold (the largest kernel instantiation).
    MAX_VECTORS_PER_THREAD = 16
    #: Widest row accepted: 8 CTAs x 512 threads x 8 vectors x 4 fp32 values.
    MAX_BLOCK_SIZE = 131072

    @staticmethod
    def max_threads_for(vectors: int) -> int:
        """Register budget per thread of each kernel instantiation (see rows.cu)."""
        return 1024 if vectors <= 4 else (512 if vectors <= 8 else 256)

    def grid(self, problem: Problem) -> Iterator[KernelConfig]:
        block = next_power_of_2(problem.dims_dict["cols"])
        yield KernelConfig(self.operation, BLOCK_SIZE=block, ROW_KERNEL=3, num_warps=1)
        for warps in self.STREAM_WARPS:
            yield KernelConfig(self.operation, BLOCK_SIZE=block, ROW_KERNEL=2, num_warps=warps)
            # two slots per row group: room for two CTAs per SM
            yield KernelConfig(self.operation, BLOCK_SIZE=block, ROW_KERNEL=2, num_warps=warps, num_stages=2)
        for cluster, warps, rows in product(self.CLUSTER, self.NUM_WARPS, self.ROWS_PER_PROGRAM):
            yield KernelConfig(
                self.operation,
                BLOCK_SIZE=block,
                ROW_KERNEL=1,
                ROWS_PER_PROGRAM=rows,
                num_warps=warps,
                CLUSTER=cluster,
            )

    #: Widest row of the warp-per-row kernel, in 16-byte vectors (4 KB).
    WARP_MAX_VECTORS = 256

    @staticmethod
    def is_stream(config: KernelConfig) -> bool:
        return config.get("ROW_KERNEL", 1) == 2

    @staticmethod
    def is_warp(config: KernelConfig) -> bool:
        return config.get("ROW_KERNEL", 1) == 3

    def vectors_per_row(self, problem: Problem) -> int:
        return ceil_div(problem.dims_dict["cols"] * problem.itemsize, 16)

    def vectors_per_thread(self, config: KernelConfig, problem: Problem) -> int:
        if self.is_warp(config):
            return ceil_div(self.vectors_per_row(problem), 32)
        if self.is_stream(config):  # interior vectors only; head/tail are scalar
            whole = problem.dims_dict["cols"] * problem.itemsize // 16
            return max(1, ceil_div(whole, config["num_warps"] * 32))
        threads = config["num_warps"] * 32 * config.get("CLUSTER", 1)
        return ceil_div(self.vectors_per_row(problem), threads)

    def num_programs(self, config: KernelConfig, problem: Problem) -> int:
        if self.is_warp(config):
            return ceil_div(problem.dims_dict["rows"], 8)
        if self.is_stream(config):
            return problem.dims_dict["rows"]
        return ceil_div(problem.dims_dict["rows"], config["ROWS_PER_PROGRAM"]) * config.get("CLUSTER", 1)

    def stream_reject_reason(self, config: KernelConfig, problem: Problem, caps: DeviceCaps) -> str | None:
        cols, rows = problem.dims_dict["cols"], problem.dims_dict["rows"]
        warps = config["num_warps"]
        if warps > self.STREAM_CONSUMER_WARPS:
            return f"streaming kernel: {warps} warps per row exceed its {self.STREAM_CONSUMER_WARPS} consumer warps"
        slot = ceil_div(cols * problem.itemsize // 16 * 16, 128) * 128
        if self.STREAM_FIXED_SMEM + slot + 8 > caps.max_shared_memory_per_block:
            return f"streaming kernel: a row of {slot} bytes does not fit one shared-memory slot"
        stages = config.get("num_stages", 0)
        if stages:
            groups = self.STREAM_CONSUMER_WARPS // warps
            need = self.STREAM_FIXED_SMEM + groups * stages * (slot + 8)
            if need > caps.max_shared_memory_per_block:
                return f"streaming kernel: {stages} row slots per group of {slot} bytes exceed shared memory"
        nv = self.vectors_per_thread(config, problem)
        if nv > self.MAX_VECTORS_PER_THREAD:
            return f"register pressure: {nv} vectors per thread"
        if warps > 1 and warps * 32 >= 2 * self.vectors_per_row(problem):
            return f"idle threads: {warps * 32} threads for {self.vectors_per_row(problem)} vectors"
        if rows < caps.sm_count:
            return f"streaming kernel: {rows} rows leave persistent CTAs of {caps.sm_count} SMs idle"
        return None

    def reject_reason(self, config: KernelConfig, problem: Problem, caps: DeviceCaps) -> str | None:
        cols, rows = problem.dims_dict["cols"], problem.dims_dict["rows"]
        if config["BLOCK_SIZE"] > self.MAX_BLOCK_SIZE:
            return f"row of {cols} exceeds the single-pass limit"
        if self.is_stream(config):
            return self.stream_reject_reason(config, problem, caps)
        if self.is_warp(config):
            if (cols * problem.itemsize) % 16 != 0:
                return "warp-per-row kernel: rows must hold whole 16-byte vectors"
            if self.vectors_per_row(problem) > self.WARP_MAX_VECTORS:
                return f"warp-per-row kernel: a row of {cols * problem.itemsize} bytes exceeds 4 KB"
            return None
        cluster = config.get("CLUSTER", 1)
        if cluster > caps.max_cluster_size:
            return f"cluster of {cluster} exceeds the portable limit of {caps.max_cluster_size}"
        threads = config["num_warps"] * caps.warp_size
        nv = self.vectors_per_thread(config, problem)
        if nv > self.MAX_VECTORS_PER_THREAD:
            return f"register pressure: {nv} vectors per thread"
        if threads > self.max_threads_for(nv):
            return f"register pressure: {nv} vectors per thread allow at most {self.max_threads_for(nv)} threads"
        idle = threads * cluster - self.vectors_per_row(problem)
        if idle >= threads * cluster // 2 and (config["num_warps"] > 1 or cluster > 1):
            return f"idle threads: {threads * cluster} threads for {self.vectors_per_row(problem)} vectors"
        if config["ROWS_PER_PROGRAM"] > rows:
            return f"ROWS_PER_PROGRAM={config['ROWS_PER_PROGRAM']} exceeds {rows} rows"
        return None

    def priority(self, config: KernelConfig, problem: Problem, caps: DeviceCaps) -> tuple[float, ...]:
        """Memory-bound: the library default first, then its kernel (streaming
        or register), then fill the machine, keep about as many 16-byte loads
        in flight per thread as the default does (eight for a softmax in
        registers, else four), prefer no cluster, then fewer rows per program."""
        from kernelo_b200.kernels.rows_common import default_rows_config

        d = problem.dims_dict
        default = default_rows_config(self.operation, d["cols"], problem.dtype, rows=d["rows"],
                                      sm_count=caps.sm_count)
        is_default = dict(config) == dict(default)
        stream_first = self.is_stream(default)
        kernel_rank = 0 if config.get("ROW_KERNEL", 1) == default.get("ROW_KERNEL", 1) else 1
        programs = min(self.num_programs(config, problem), caps.sm_count)
        nv = self.vectors_per_thread(config, problem)
        target = 3 if (self.operation == "softmax" and not stream_first) else 2
        return (0 if is_default else 1, kernel_rank, -programs, abs(math.log2(nv) - target),
                config.get("CLUSTER", 1), config.get("ROWS_PER_PROGRAM", 1))


class SoftmaxSearchSpace(_RowReductionSpace):
    operation = "softmax"


class RMSNormSearchSpace(_RowReductionSpace):
    operation = "rmsnorm"


SEARCH_SPACES: dict[str, type[SearchSpace]] = {
    "softmax": SoftmaxSearchSpace,
    "matmul": MatmulSearchSpace,
    "rmsnorm": RMSNormSearchSpace,
    "fused_linear": FusedLinearSearchSpace,
    "fused_linear_erf": FusedLinearErfSearchSpace,
    "gemv": GemvSearchSpace,
}


def search_space(operation: str, **kwargs) -> SearchSpace:
    try:
        return SEARCH_SPACES[operation](**kwargs)
    except KeyError:
        raise ValueError(f"no search space for {operation!r}; known: {sorted(SEARCH_SPACES)}") from None
