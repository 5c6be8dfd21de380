"""Candidate generation for sm_100a (``kernelforge/tuning/search.py:1-558``).

Same three stages as the reference -- enumerate a grid, reject points with a
named reason, budget the survivors by a documented priority -- over the
parameters that matter on Blackwell instead of Triton's:

GEMM (``matmul``, ``fused_linear``, ``fused_linear_erf``, ``gemv``)
    tcgen05 grid: MMA tile ``BLOCK_M`` {64, 128, 256 (2-CTA pair)} x ``BLOCK_N``
    {16, 64, 128, 192, 256} x ``BLOCK_K`` {32, 64, 128} x ``num_stages``
    (shared-memory ring depth) {2, 4, 6} x thread-block cluster
    {1x1, 2x1, 1x2, 2x2} = 540 points, plus the 3 SIMT tiles that serve fp32
    and operands no TMA tensor map can describe. ``SWAP_AB`` is derived from
    the shape (skinny M puts the weight on the 128-row side) and ``STREAM_K``
    is left to the library (stream-K when whole tiles would leave SMs idle).

    Hardware limits: 227 KiB shared memory per CTA, 512 TMEM columns per SM
    (a double-buffered fp32 accumulator needs 2 x BLOCK_N), TMA's 16-byte
    stride rule, whole 128-byte swizzle atoms (BLOCK_K >= 64 for 16-bit), an
    MN-major B operand taking 64-column boxes. Implementation limits of this
    build are rejected with "not implemented" so they stay visible.

Row reductions (``softmax``, ``rmsnorm``)
    ``num_warps`` {1..32} x ``ROWS_PER_PROGRAM`` {1, 2, 4} x ``CLUSTER``
    {1, 2, 4, 8} (CTAs sharing one row through distributed shared memory).
    ``BLOCK_SIZE`` (next power of two of the row) is kept for the reference's
    "cannot hold a row" / "single-pass limit" checks; the single-pass limit
    rises from 16384 to 131072 columns because a row may span a cluster.

Filters read a :class:`DeviceCaps` value, never ``torch.cuda``, so they are
unit-testable without the GPU they describe.
"""

from __future__ import annotations

import math
from abc import ABC, abstractmethod
from collections.abc import Iterator
from itertools import product

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


class SearchSpace(ABC):
    """Configurations worth trying for one operation."""

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
        raise NotImplementedError

    def priority(self, config: KernelConfig, problem: Problem, caps: DeviceCaps) -> tuple[float, ...]:
        """Budget sort key, lower first (ties broken by the serialised config)."""
        return (0.0,)

    def candidates(
        self, problem: Problem, caps: DeviceCaps | None = None, *, max_candidates: int | None = None
    ) -> list[KernelConfig]:
        return self.generate(problem, caps, max_candidates=max_candidates).candidates

    def generate(
        self, problem: Problem, caps: DeviceCaps | None = None, *, max_candidates: int | None = None
    ) -> CandidateSet:
        if problem.operation != self.operation:
            raise ValueError(
                f"{type(self).__name__} handles {self.operation!r}, got {problem.operation!r}"
            )
        caps = caps if caps is not None else device_caps()
        budget = max_candidates if max_candidates is not None else self.max_candidates
        kept: list[KernelConfig] = []
        rejected: list[tuple[KernelConfig, str]] = []
        generated = 0
        for config in self.grid(problem):
            generated += 1
            why = self.reject_reason(config, problem, caps)
            if why is None:
                kept.append(config)
            else:
                rejected.append((config, why))
        feasible = len(kept)
        kept, pruned = self._prune_underutilised(kept, problem, caps)
        rejected.extend(pruned)
        kept.sort(key=lambda c: (*self.priority(c, problem, caps), c.to_json()))
        return CandidateSet(
            problem=problem,
            generated=generated,
            feasible=feasible,
            after_prune=len(kept),
            budget=budget,
            candidates=kept[:budget],
            rejected=tuple(rejected),
        )

    def _prune_underutilised(
        self, configs: list[KernelConfig], problem: Problem, caps: DeviceCaps
    ) -> tuple[list[KernelConfig], list[tuple[KernelConfig, str]]]:
        """Drop configs whose launch fills under half the SMs -- unless none can fill them all."""
        try:
            programs = {c: self.num_programs(c, problem) for c in configs}
        except NotImplementedError:
            return configs, []
        if not programs or max(programs.values()) < caps.sm_count:
            return configs, []
        floor = caps.sm_count // 2
        kept = [c for c in configs if programs[c] >= floor]
        dropped = [
            (c, f"launch grid of {programs[c]} programs fills under half of {caps.sm_count} SMs")
            for c in configs
            if programs[c] < floor
        ]
        return kept, dropped

    def explain(self, problem: Problem, caps: DeviceCaps | None = None) -> str:
        resolved = caps if caps is not None else device_caps()
        result = self.generate(problem, resolved)
        suffix = "" if resolved.measured else "  <- no device attached"
        lines = [
            problem.describe(),
            f"  device           : {resolved.name}, {resolved.sm_count} SMs, "
            f"{resolved.max_shared_memory_per_block // 1024} KiB shared/block{suffix}",
            f"  grid points      : {result.generated}",
            f"  feasible         : {result.feasible}",
            f"  after prune      : {result.after_prune}",
            f"  selected (budget): {len(result.candidates)} of {result.budget}",
        ]
        counts: dict[str, int] = {}
        for _, reason in result.rejected:
            rule = reason.split(":")[0].split("(")[0].strip()
            counts[rule] = counts.get(rule, 0) + 1
        if counts:
            lines.append("  rejections by rule:")
            lines.extend(f"    {n:>4}  {rule}" for rule, n in sorted(counts.items(), key=lambda kv: -kv[1]))
        return "\n".join(lines)


class CandidateSet:
    """Candidates plus the count left after each stage."""

    __slots__ = ("problem", "generated", "feasible", "after_prune", "budget", "candidates", "rejected")

    def __init__(self, *, problem, generated, feasible, after_prune, budget, candidates, rejected):
        self.problem = problem
        self.generated = generated
        self.feasible = feasible
        self.after_prune = after_prune
        self.budget = budget
        self.candidates = candidates
        self.rejected = rejected

    def __len__(self) -> int:
        return len(self.candidates)

    def __iter__(self) -> Iterator[KernelConfig]:
        return iter(self.candidates)


# ------------------------------------------------------------------------ GEMM
class _Sm100GemmSpace(SearchSpace):
    """tcgen05 tile grid plus the SIMT fallback tiles, shared by the GEMM operators."""

    BLOCK_M = (64, 128, 256)
    BLOCK_N = (16, 64, 128, 192, 256)
    BLOCK_K = (32, 64, 128)
    NUM_STAGES = (2, 3, 4, 6)
    CLUSTERS = ((1, 1), (2, 1), (1, 2), (2, 2))
    #: L2 the A panels of one raster group may take (the library default's rule).
    GROUP_L2_BYTES = 48 << 20
    #: (BLOCK_M, BLOCK_N, BLOCK_K) of the CUDA-core kernel's instantiations.
    SIMT_TILES = ((128, 128, 8), (64, 64, 16), (128, 64, 16))
    #: How B is laid out for this operator's canonical inputs.
    b_layout = "nk"

    def dims(self, problem: Problem) -> tuple[int, int, int]:
        d = problem.dims_dict
        return d["M"], d["N"], d["K"]

    def group_m(self, block_m: int, problem: Problem) -> int:
        """Raster group width: as many M tiles as keep their A panels within
        GROUP_L2_BYTES of L2 (so each group streams B once)."""
        m, n, k = self.dims(problem)
        m_k = n if gc.default_swap(m, n) else m
        rows = max(block_m, gc.TC_BLOCK_M)
        return max(1, min(ceil_div(m_k, rows), self.GROUP_L2_BYTES // max(1, rows * k * problem.itemsize)))

    def library_default(self, problem: Problem) -> KernelConfig:
        """The config the library picks on its own: always a candidate, so that
        tuning never ends worse than not tuning."""
        m, n, k = self.dims(problem)
        return gc.default_gemm_config(self.operation, m, n, k, problem.dtype, b_layout=self.b_layout)

    def grid(self, problem: Problem) -> Iterator[KernelConfig]:
        default = self.library_default(problem)
        yield default
        for config in self._grid(problem):
            if config != default:
                yield config

    def _grid(self, problem: Problem) -> Iterator[KernelConfig]:
        m, n, _ = self.dims(problem)
        if self.b_layout == "nk":
            # decode shapes: 16-row weight tiles on mma.sync (BLOCK_M warps per tile,
            # num_stages vector pairs in flight)
            for warps, pairs in gc.TILE_ROWS_SHAPES:
                yield KernelConfig(self.operation, KERNEL=gc.KERNEL_TILE_ROWS, BLOCK_M=warps, num_stages=pairs)
        swap = 1 if gc.default_swap(m, n) else 2
        for bm, bn, bk, stages, (cm, cn) in product(
            self.BLOCK_M, self.BLOCK_N, self.BLOCK_K, self.NUM_STAGES, self.CLUSTERS
        ):
            yield KernelConfig(
                self.operation,
                KERNEL=gc.KERNEL_TCGEN05,
                BLOCK_M=bm,
                BLOCK_N=bn,
                BLOCK_K=bk,
                GROUP_M=self.group_m(bm, problem),
                num_stages=stages,
                STREAM_K=0,
                SWAP_AB=swap,
                CLUSTER_M=cm,
                CLUSTER_N=cn,
            )
        for bm, bn, bk in self.SIMT_TILES:
            yield KernelConfig(self.operation, KERNEL=gc.KERNEL_SIMT, BLOCK_M=bm, BLOCK_N=bn, BLOCK_K=bk)

    def kernel_view(self, config: KernelConfig, problem: Problem) -> tuple[int, int]:
        """(M', N') the kernel tiles, after an A/B swap."""
        m, n, _ = self.dims(problem)
        if config.get("SWAP_AB", 2) == 1:
            return n, m
        return m, n

    def shared_memory_bytes(self, config: KernelConfig, problem: Problem) -> int:
        if config["KERNEL"] == gc.KERNEL_TILE_ROWS:
            m = self.dims(problem)[0]
            return (config["BLOCK_M"] - 1) * 32 * gc.tile_rows_groups(m) * 16  # the K-slice partials
        if config["KERNEL"] == gc.KERNEL_SIMT:
            return 2 * config["BLOCK_K"] * (config["BLOCK_M"] + config["BLOCK_N"]) * 4
        return gc.tc_smem_bytes(config["BLOCK_N"], config["BLOCK_K"], config["num_stages"],
                                itemsize(problem.dtype), gc.cta_group(config["BLOCK_M"]))

    def num_programs(self, config: KernelConfig, problem: Problem) -> int:
        """CTAs with work: tiles, times two for SM-pair tiles."""
        if config["KERNEL"] == gc.KERNEL_TILE_ROWS:
            return ceil_div(self.dims(problem)[1], 16)  # one CTA per 16 weight rows
        m_k, n_k = self.kernel_view(config, problem)
        tiles = ceil_div(m_k, config["BLOCK_M"]) * ceil_div(n_k, config["BLOCK_N"])
        return tiles * (gc.cta_group(config["BLOCK_M"]) if config["KERNEL"] == gc.KERNEL_TCGEN05 else 1)

    def reject_reason(self, config: KernelConfig, problem: Problem, caps: DeviceCaps) -> str | None:
        m, n, k = self.dims(problem)
        if config["KERNEL"] == gc.KERNEL_TILE_ROWS:
            return gc.tile_rows_reject(m, k, problem.dtype)
        if config["KERNEL"] == gc.KERNEL_SIMT:
            return None  # the fallback always runs
        why = gc.shape_allows_tcgen05(m, n, k, problem.dtype, b_layout=self.b_layout)
        if why is not None:
            return why
        bm, bn, bk, stages = config["BLOCK_M"], config["BLOCK_N"], config["BLOCK_K"], config["num_stages"]
        cluster = (config["CLUSTER_M"], config["CLUSTER_N"])
        if bm == 64:
            return "not implemented: BLOCK_M=64 (M=64 MMAs use a different TMEM layout)"
        cg = gc.cta_group(bm)
        if cg == 2 and cluster != (2, 1):
            if cluster == (1, 1):
                return "SM pair: BLOCK_M=256 runs on a 2x1 cluster (CLUSTER_M=2)"
            return f"not implemented: cluster {cluster[0]}x{cluster[1]} beyond the SM pair"
        if cg == 1 and cluster != (1, 1):
            return (f"not implemented: cluster {cluster[0]}x{cluster[1]} without the pair MMA "
                    "(sharing tiles would need TMA multicast)")
        if bn % (16 * cg) != 0:
            return f"SM pair: BLOCK_N={bn} does not split into two 16-column halves"
        if bk * itemsize(problem.dtype) < 128:
            return f"swizzle atom: BLOCK_K={bk} is less than one 128-byte swizzle row"
        smem = self.shared_memory_bytes(config, problem)
        if smem > caps.max_shared_memory_per_block:
            return (
                f"shared memory: {smem // 1024} KiB of tiles exceeds the "
                f"{caps.max_shared_memory_per_block // 1024} KiB per-block limit"
            )
        tmem = gc.tc_tmem_columns(bn)
        if tmem > caps.tmem_columns_per_sm:
            return f"TMEM: {tmem} accumulator columns exceed {caps.tmem_columns_per_sm} per SM"
        swapped = config["SWAP_AB"] == 1
        if self.b_layout == "kn" and not swapped and (bn // cg) % 64 != 0:
            return f"MN-major B: BLOCK_N={bn} gives each CTA a share that is not 64-column TMA boxes"
        m_k, n_k = self.kernel_view(config, problem)
        smallest = min(v for v in self.BLOCK_N if self.b_layout != "kn" or swapped or v % 64 == 0)
        if bn > 2 * n_k and bn > smallest:
            return f"tile overshoot: BLOCK_N={bn} for N={n_k}"
        if cg == 2 and m_k <= gc.TC_BLOCK_M:
            return f"tile overshoot: BLOCK_M={bm} for M={m_k}"
        k_iters = ceil_div(k, bk)
        if stages > 2 and k_iters < stages:
            return f"pipeline cannot fill: {k_iters} K iterations for num_stages={stages}"
        return None

    def priority(self, config: KernelConfig, problem: Problem, caps: DeviceCaps) -> tuple[float, ...]:
        """The tile kernel first where it runs (its default shape first); then
        tcgen05 before SIMT; then parallelism up to one wave; then reuse
        BM*BN/(BM+BN) (operand bytes per MMA); then least padding; then the
        deeper ring."""
        if config == self.library_default(problem):
            return (-10,)
        if config["KERNEL"] == gc.KERNEL_TILE_ROWS:
            default = (config["BLOCK_M"], config["num_stages"]) == gc.tile_rows_default(self.dims(problem)[0])
            return (-3,) if default else (-2,)
        kernel_rank = 0 if config["KERNEL"] == gc.KERNEL_TCGEN05 else 1
        m_k, n_k = self.kernel_view(config, problem)
        bm, bn = config["BLOCK_M"], config["BLOCK_N"]
        programs = min(self.num_programs(config, problem), caps.sm_count)
        reuse = bm * bn / (bm + bn)
        padded = ceil_div(m_k, bm) * bm * ceil_div(n_k, bn) * bn
        waste = padded / (m_k * n_k)
        return (kernel_rank, -programs, -reuse, waste, -config.get("num_stages", 0))


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
    warps per row group, one CTA per SM with 16 consumer warps."""

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

    @staticmethod
    def is_stream(config: KernelConfig) -> bool:
        return config.get("ROW_KERNEL", 1) == 2

    def vectors_per_row(self, problem: Problem) -> int:
        return ceil_div(problem.dims_dict["cols"] * problem.itemsize, 16)

    def vectors_per_thread(self, config: KernelConfig, problem: Problem) -> int:
        if self.is_stream(config):  # interior vectors only; head/tail are scalar
            whole = problem.dims_dict["cols"] * problem.itemsize // 16
            return max(1, ceil_div(whole, config["num_warps"] * 32))
        threads = config["num_warps"] * 32 * config.get("CLUSTER", 1)
        return ceil_div(self.vectors_per_row(problem), threads)

    def num_programs(self, config: KernelConfig, problem: Problem) -> int:
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
        kernel_rank = 0 if self.is_stream(config) == stream_first else 1
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
