"""Shared host logic of the GEMM-shaped operators (matmul, fused_linear, gemv).

Mirrors, in Python, the two decisions the native library makes per call so
that configs can be stated explicitly (cached, ranked, filtered):

* whether an operand can be described by a TMA tensor map (16-byte aligned
  base, unit stride along K or along M/N, the other stride a multiple of 16
  bytes) -- otherwise a 16-bit problem that is not skinny is packed into the
  workspace for tcgen05, and the rest go to the SIMT kernel;
* the default tcgen05 tile for a shape: 256-row SM-pair tiles when they fill
  the machine (else 128-row), BLOCK_N up to 256, A/B swapped for skinny M (the
  weight becomes the 128-row operand), all stream-K when whole tiles would
  leave SMs idle, else the split tail (whole tiles, the last partial wave as
  half-width tiles).
"""

from __future__ import annotations

import torch

from kernelo_b200.tuning.config import KernelConfig

KERNEL_TCGEN05 = 1
KERNEL_SIMT = 2
#: kf_gemv only: warps streaming K-contiguous weight rows, M <= 4 (csrc/gemv_rows.cu).
KERNEL_WARP_ROWS = 3
#: kf_gemv's 16-row weight tiles on mma.sync (fp16/bf16, M <= 32, K % 8 == 0);
#: BLOCK_M = warps per tile (K slices), num_stages = vector pairs in flight.
KERNEL_TILE_ROWS = 4
TILE_ROWS_MAX_M = 32
#: kf_gemm / kf_gemv: lanes streaming an N-contiguous B's rows (the row-major
#: (K, N) operand), M <= 8, any dtype, K split over CTAs (csrc/gemv_cols.cu).
KERNEL_COLUMNS = 5
COLUMNS_MAX_M = 8
#: kf_gemv / kf_gemm: the 16-row tile GEMV with the weight streamed through a shared-memory
#: ring of bulk copies, one persistent CTA per SM (fp16/bf16, M <= 16, K % 8 == 0; no peers);
#: num_stages = ring depth (0: as deep as fits), NUM_CTAS = grid (csrc/gemv_stream.cu).
KERNEL_TILE_STREAM = 6
TILE_STREAM_MAX_M = 16
#: weight elements per row per ring stage (BLOCK_K) compiled in gemv_stream.cu; the first is the default
TILE_STREAM_CHUNKS = (1024, 512)
#: (warps per tile, vector pairs per batch; 1 = one software-pipelined pair) compiled in gemv_mma.cu
TILE_ROWS_SHAPES = ((8, 1), (8, 2), (8, 4), (6, 2), (6, 4), (4, 2), (4, 4), (4, 8))


def tile_rows_groups(m: int) -> int:
    """8-row groups of x the kernel is compiled for (mirrors gemv_mma.cu)."""
    return 1 if m <= 8 else (2 if m <= 16 else 4)


def tile_rows_default(m: int) -> tuple[int, int]:
    """The kernel's default shape (mirrors gemv_mma.cu)."""
    return {1: (8, 1), 2: (6, 4), 4: (4, 4)}[tile_rows_groups(m)]


def tile_rows_split(n: int, m: int = 1, sm_count: int = 148) -> int:
    """CTAs per 16-row weight tile the tile GEMV uses by default (mirrors
    default_tile_split in gemv_mma.cu): the fewest of 1, 2, 4 that give at
    least two CTAs per SM up to 8 rows of x, four beyond, the tile's K split
    over a thread-block cluster."""
    tiles = -(-n // 16)
    target = (2 if m <= 8 else 4) * sm_count
    ks = 1
    while ks < 4 and tiles * ks < target:
        ks *= 2
    return ks


def tile_stream_preferred(m: int, n: int, k: int, *, sm_count: int = 148, overlap: bool = False) -> bool:
    """Whether the library runs a supported decode shape on the streamed tile
    kernel rather than the register-fed one (mirrors gemv_stream_preferred in
    kf_internal.h). Without overlap: beyond 8 rows of x when K is long or the
    16-row tiles number at least eight per SM. With overlap: beyond 8 rows,
    for long K, or below four tiles per SM."""
    if not 1 <= m <= TILE_STREAM_MAX_M:
        return False
    tiles = -(-n // 16)
    if overlap:
        return m > 8 or k >= 8192 or tiles < 4 * sm_count
    return m > 8 and (k >= 8192 or tiles >= 8 * sm_count)


def tile_stream_reject(m: int, k: int, dtype: torch.dtype) -> str | None:
    """Why the streamed tile GEMV cannot take this contiguous problem (None: it can)."""
    if not 1 <= m <= TILE_STREAM_MAX_M:
        return f"the streamed tile GEMV takes 1..{TILE_STREAM_MAX_M} rows of x, got M={m}"
    return tile_rows_reject(m, k, dtype)


def tile_stream_smem_bytes(m: int, chunk: int, max_smem: int = 232448) -> int:
    """Shared memory of the streamed tile GEMV at its default ring depth (mirrors launch_gemv_stream)."""
    stage = 16 * chunk * 2
    # alignment slack, the two-slot x ring and its barriers, the warps' partial tiles, two flags
    fixed = 128 + 2 * (stage + 16) + 8 * 32 * (1 if m <= 8 else 2) * 16 + 16
    stages = min(12, (max_smem - fixed) // (stage + 16))
    return fixed + stages * (stage + 16)


def tile_rows_reject(m: int, k: int, dtype: torch.dtype) -> str | None:
    """Why the tile GEMV cannot take this contiguous problem (None: it can)."""
    if dtype not in (torch.float16, torch.bfloat16):
        return "the tile GEMV takes fp16 or bf16"
    if not 1 <= m <= TILE_ROWS_MAX_M:
        return f"the tile GEMV takes 1..{TILE_ROWS_MAX_M} rows of x, got M={m}"
    if k % 8 != 0:
        return "the tile GEMV needs K % 8 == 0 (whole 16-byte vectors)"
    return None
def columns_reject(m: int, n: int, k: int, dtype: torch.dtype, *, b_layout: str) -> str | None:
    """Why the column GEMV cannot take this contiguous problem (None: it can;
    mirrors gemv_cols_supported in gemv_cols.cu)."""
    if b_layout != "kn":
        return "the column GEMV streams an N-contiguous B (a row-major (K, N) operand)"
    if not 1 <= m <= COLUMNS_MAX_M:
        return f"the column GEMV takes 1..{COLUMNS_MAX_M} rows of x, got M={m}"
    ve = 16 // torch.empty(0, dtype=dtype).element_size()
    if n % ve != 0 or k < 1:
        return f"the column GEMV needs N a multiple of {ve} (whole 16-byte vectors)"
    return None


def columns_programs(n: int, k: int, dtype: torch.dtype, sm_count: int = 148) -> int:
    """CTAs of the column GEMV: 32-vector column strips times the K split
    (mirrors gemv_cols_splits)."""
    ve = 16 // torch.empty(0, dtype=dtype).element_size()
    strips = -(-n // (32 * ve))
    splits = max(1, min(-(-4 * sm_count // strips), max(1, k // 64), 256))
    return strips * splits


WARP_ROWS_MAX_M = 4
#: The library default up to this M (measured on B200: at M=4 the tcgen05 GEMV is faster).
WARP_ROWS_AUTO_MAX_M = 2


def warp_rows_rows(m: int) -> int:
    """Rows of x the warp-per-row GEMV is compiled for: M rounded up to 1, 2 or 4."""
    return 1 if m <= 1 else 2 if m <= 2 else 4


def warp_rows_smem_bytes(m: int, k: int, itemsize: int = 2) -> int:
    """x staged as fp32: whole 16-byte weight vectors plus one vector of tail."""
    ve = 16 // itemsize
    return warp_rows_rows(m) * (k // ve * ve + ve) * 4

SM100_SMEM_PER_BLOCK = 232_448
SM100_SMS = 148
TC_BLOCK_M = 128
#: Bytes the kernel adds to its operand ring: alignment slack and barriers.
TC_SMEM_OVERHEAD = 1024 + 8 * 37 + 16


def tc_smem_bytes(block_n: int, block_k: int, stages: int, itemsize: int = 2, cta_group: int = 1) -> int:
    """Shared memory of one tcgen05 CTA: the A/B ring plus barriers.

    Each CTA stages 128 rows of A and its share of B: all BLOCK_N rows for a
    one-SM tile, half of them for a 256-row SM-pair tile.
    """
    # fp32 (TF32-split) stages hold both parts of every element
    stage_bytes = 2 * itemsize if itemsize == 4 else itemsize
    ring = stages * (TC_BLOCK_M + block_n // cta_group) * block_k * stage_bytes
    return ring + 1024 + 8 * (2 * stages + 5) + 16


def cta_group(block_m: int) -> int:
    """SMs per MMA: BLOCK_M=256 tiles run on an SM pair (tcgen05 cta_group::2)."""
    return 2 if block_m == 2 * TC_BLOCK_M else 1


def tc_tmem_columns(block_n: int) -> int:
    """TMEM columns: a double-buffered fp32 accumulator, rounded to a power of two >= 32."""
    cols = 32
    while cols < 2 * block_n:
        cols *= 2
    return cols


def operand_major(t: torch.Tensor, mn_dim: int, k_dim: int) -> int:
    """0 = K-major, 1 = MN-major, -1 = no TMA description (mirrors gemm_tcgen05.cu)."""
    if t.dtype not in (torch.float16, torch.bfloat16):
        return -1
    if t.data_ptr() % 16 != 0:
        return -1
    mn, k = t.shape[mn_dim], t.shape[k_dim]
    s_mn, s_k = t.stride(mn_dim), t.stride(k_dim)
    if k < 8:
        return -1
    if s_k == 1 and (mn == 1 or (s_mn % 8 == 0 and s_mn >= k)):
        return 0
    if s_mn == 1 and s_k % 8 == 0 and s_k >= mn:
        return 1
    return -1


def tma_misfit(m: int, n: int, k: int, *, b_layout: str) -> str | None:
    """Why contiguous operands of this shape cannot be TMA tensor maps as they
    are (mirrors operand_major in gemm_tcgen05.cu), or None.

    ``b_layout`` is ``"kn"`` for a row-major (K, N) B (matmul) and ``"nk"`` for
    an nn.Linear-style [N, K] weight.
    """
    if k < 8:
        return f"TMA alignment: K={k} is below one 16-byte vector"
    if m > 1 and k % 8 != 0:
        return f"TMA alignment: A row stride K={k} is not a multiple of 16 bytes"
    if b_layout == "kn" and n > 1 and n % 8 != 0:
        return f"TMA alignment: B row stride N={n} is not a multiple of 16 bytes"
    if b_layout == "nk" and n > 1 and k % 8 != 0:
        return f"TMA alignment: W row stride K={k} is not a multiple of 16 bytes"
    return None


def packs_by_default(m: int, n: int, k: int, dtype: torch.dtype, *, b_layout: str) -> bool:
    """Whether the library packs this problem's operands for tcgen05 on its own
    (mirrors packing_applies in api.cu): 16-bit operands TMA cannot describe,
    in a problem that is not skinny (M and N above 64)."""
    return (dtype in (torch.float16, torch.bfloat16) and k > 0 and m > 64 and n > 64
            and tma_misfit(m, n, k, b_layout=b_layout) is not None)


def shape_allows_tcgen05(m: int, n: int, k: int, dtype: torch.dtype, *, b_layout: str) -> str | None:
    """Why operands of this shape cannot take the tcgen05 path, or None. Any
    16-bit layout can: operands TMA cannot describe are first packed into the
    workspace as pitched copies (csrc/pack.cu); fp32 operands are split into
    K-major TF32 parts (csrc/tf32_split.cu) and run as 3xTF32 on kind::tf32."""
    if dtype not in (torch.float16, torch.bfloat16, torch.float32):
        return "tcgen05 takes fp16/bf16 (kind::f16) or fp32 as 3xTF32 (kind::tf32)"
    return None


def default_swap(m: int, n: int) -> bool:
    return m <= 64 and n > m


def tf32_split_k(k: int) -> int:
    """The K the tcgen05 kernel sees for an fp32 problem: K rounded up to a
    32-element atom; each k-block carries both TF32 parts (mirrors tf32_split.cu)."""
    return -(-k // 32) * 32


def tf32_applies(m: int, n: int, k: int, dtype: torch.dtype) -> bool:
    """fp32 runs as 3xTF32 on tensor cores by default when both M and N exceed 64
    and the problem has at least 2^27 multiply-adds (mirrors tf32_applies in api.cu)."""
    return dtype == torch.float32 and k > 0 and m > 64 and n > 64 and m * n * k >= 1 << 27


def default_tcgen05_config(
    operation: str, m: int, n: int, k: int, *, b_layout: str, sm_count: int = 148, elem: int = 2
) -> KernelConfig:
    """The tcgen05 config the library would choose for contiguous operands of
    ``elem``-byte elements (4: the TF32-split fp32 operands, K the split K)."""
    swap = default_swap(m, n)
    m_k, n_k = (n, m) if swap else (m, n)
    # B' (the kernel's second operand) is MN-major for matmul's row-major B
    # unless swapped (then B' is A, which is K-major).
    b_mn = (b_layout == "kn") and not swap
    pair_tiles = -(-m_k // 256) * -(-n_k // 256)
    cg = 2 if (m_k >= 256 and n_k >= 128 and pair_tiles >= sm_count // 2) else 1
    quantum = (64 if b_mn else 16) * cg
    widest = 128 if elem == 4 else 256  # TF32 tiles sum their chunks in registers
    if n_k <= widest:
        block_n = max(quantum, -(-n_k // quantum) * quantum)
    else:
        block_n = widest
    atom = 128 // elem  # elements per 128-byte swizzle row
    stage_elem = 2 * elem if elem == 4 else elem  # TF32 stages carry both split parts
    block_k = 2 * atom if (cg == 2 and k >= 512) else atom
    per_stage = (TC_BLOCK_M + block_n // cg) * block_k * stage_elem
    stages = max(2, min(12, (SM100_SMEM_PER_BLOCK - 1024 - 256) // per_stage))
    tiles_m = -(-m_k // (TC_BLOCK_M * cg))
    tiles = tiles_m * -(-n_k // block_n)
    k_blocks = -(-k // block_k)
    # (mirrors api.cu) short K: whole tiles; below one wave of one-SM tiles,
    # stream-K for a long K and narrower whole tiles for a short one; else the split tail
    if k_blocks < 4:
        stream_k = 2
    elif cg == 1 and tiles < sm_count and (k_blocks < 16 or tiles * k_blocks < 8 * sm_count):
        quantum = 64 if b_mn else 16
        for bn in (128, 64):
            if tiles >= sm_count or bn >= block_n or bn % quantum:
                continue
            block_n = bn
            tiles = tiles_m * -(-n_k // bn)
        stream_k = 2
    else:
        stream_k = 1 if (cg == 1 and tiles < sm_count) else 3
    # A panels of one raster group within ~48 MB of L2 (mirrors api.cu)
    tile_rows = TC_BLOCK_M * cg
    group_m = max(1, min(-(-m_k // tile_rows), (48 << 20) // max(1, tile_rows * k * stage_elem)))
    return KernelConfig(
        operation,
        KERNEL=KERNEL_TCGEN05,
        BLOCK_M=TC_BLOCK_M * cg,
        BLOCK_N=block_n,
        BLOCK_K=block_k,
        GROUP_M=group_m,
        num_stages=stages,
        STREAM_K=stream_k,
        SWAP_AB=1 if swap else 2,
        CLUSTER_M=cg,
        CLUSTER_N=1,
    )


def default_simt_config(operation: str, m: int, n: int, *, sm_count: int = 148) -> KernelConfig:
    small = m * n < 128 * 128 * sm_count
    if small:
        return KernelConfig(operation, KERNEL=KERNEL_SIMT, BLOCK_M=64, BLOCK_N=64, BLOCK_K=16)
    return KernelConfig(operation, KERNEL=KERNEL_SIMT, BLOCK_M=128, BLOCK_N=128, BLOCK_K=8)


def default_gemm_config(
    operation: str, m: int, n: int, k: int, dtype: torch.dtype, *, b_layout: str, sm_count: int = 148
) -> KernelConfig:
    """The library's choice for contiguous operands (mirrors gemm_common in api.cu): the 16-row
    tile kernel for up to 32 rows of x against a K-contiguous B, the column GEMV for up to 8
    rows against an N-contiguous B, fp32 beyond 64 x 64 as 3xTF32 tcgen05 tiles, else tcgen05
    tiles (operands TMA cannot describe packed first when the problem is not skinny), else the
    CUDA-core kernel."""
    if b_layout == "nk" and tile_stream_reject(m, k, dtype) is None and tile_stream_preferred(
            m, n, k, sm_count=sm_count):
        return KernelConfig(operation, KERNEL=KERNEL_TILE_STREAM, BLOCK_K=TILE_STREAM_CHUNKS[0])
    if b_layout == "nk" and tile_rows_reject(m, k, dtype) is None:
        warps, pairs = tile_rows_default(m)
        return KernelConfig(operation, KERNEL=KERNEL_TILE_ROWS, BLOCK_M=warps, num_stages=pairs)
    if columns_reject(m, n, k, dtype, b_layout=b_layout) is None:
        return KernelConfig(operation, KERNEL=KERNEL_COLUMNS)
    if tf32_applies(m, n, k, dtype):
        # both operands split into K-major TF32 parts first
        return default_tcgen05_config(operation, m, n, tf32_split_k(k), b_layout="nk", sm_count=sm_count, elem=4)
    if dtype in (torch.float16, torch.bfloat16) and tma_misfit(m, n, k, b_layout=b_layout) is None:
        return default_tcgen05_config(operation, m, n, k, b_layout=b_layout, sm_count=sm_count)
    if packs_by_default(m, n, k, dtype, b_layout=b_layout):
        # the packed copies keep each operand's unit-stride dimension innermost,
        # with K padded to at least 8
        return default_tcgen05_config(operation, m, n, max(k, 8), b_layout=b_layout, sm_count=sm_count)
    return default_simt_config(operation, m, n, sm_count=sm_count)
