// Persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
//   C[M,N] = epilogue(A[M,K] . B[K,N])       fp16/bf16 in, fp32 accumulate
//
// and, with T = float, the same on TF32 operands (kind::tf32): the fp32 GEMM's
// split operands (tf32_split.cu), K-major, whose extended K holds the three
// partial products of the 3xTF32 scheme.
//
// One CTA per SM, 6 warps:
//   warp 0      TMA producer: 2-D tiled bulk loads of A and B k-blocks into a
//               `stages`-deep ring of 128-byte-swizzled shared-memory tiles,
//               completion tracked by full/empty mbarrier pairs.
//   warp 1      allocates TMEM, then one lane issues tcgen05.mma into a
//               double-buffered fp32 accumulator in TMEM and releases ring
//               slots with tcgen05.commit.
//   warps 2-5   epilogue: tcgen05.ld the accumulator (each warp owns one
//               32-lane TMEM quadrant = 32 rows), add bias, apply GELU, round
//               to the output dtype and store -- while the MMA warp already
//               accumulates the next tile into the other TMEM buffer.
//
// Two tile shapes, chosen by the template parameter CG (CTAs per MMA):
//   CG = 1   one SM computes a 128 x BN tile with M=128 MMAs.
//   CG = 2   a thread-block cluster of two SMs computes a 256 x BN tile with
//            the pair MMA (tcgen05.mma.cta_group::2, M=256): each CTA stages
//            its own 128 rows of A and half (BN/2 rows) of B, so per SM the
//            tensor core reads half the B bytes it would read for a 128 x BN
//            tile -- the shared-memory bandwidth a 1-SM 128x256 tile runs out
//            of. Both CTAs' TMA loads complete on the leader CTA's barrier,
//            only the leader issues MMAs, and its commits arrive on both
//            CTAs' barriers; each CTA's epilogue drains its own TMEM half.
//
// Operands may be K-major or MN-major in global memory (row-major (K,N) B,
// nn.Linear's [N,K] weight and transposed views all map to a TMA tensor map
// without a copy); the MMA reads either layout through its smem descriptors.
//
// Work is a list of segments (tile, k-block range). Data-parallel mode gives
// every CTA (pair) whole tiles in a grouped (GROUP_M) raster. Stream-K mode
// (the library picks it for one-SM tiles; pairs run it when asked) splits the
// flattened (tile, k-block) iteration space evenly over the grid; a tile
// split between units is finished by whichever
// contributor arrives last, which sums the fp32 partials in a fixed order (so
// results are deterministic) and runs the epilogue. Nobody waits for another
// CTA, so the scheme cannot deadlock.
//
// Reference: kernelforge/kernels/matmul.py:54-113 (blocked GEMM with grouped
// ordering) and kernelforge/kernels/fused_linear.py:49-104 (bias + GELU in the
// epilogue). The algorithm (tile, accumulate in fp32, fused epilogue) is the
// same; the mechanics are Blackwell's.
#include <cudaTypedefs.h>

#include <map>
#include <mutex>
#include <tuple>

#include "kf_common.cuh"
#include "kf_internal.h"

namespace kf {
namespace {

constexpr int BM = 128;  // rows per CTA (the TMEM lane count)
// Warp 0 TMA, warp 1 MMA, warps 2-9 epilogue: two epilogue warps per TMEM lane
// quadrant, each draining half of the tile's columns, so the bias + GELU
// epilogue keeps up with the pair MMA's mainloop.
constexpr int EPI_WARP0 = 2;
constexpr int NUM_EPI_WARPS = 8;
constexpr int NUM_EPI_THREADS = NUM_EPI_WARPS * 32;
constexpr int NUM_THREADS = (EPI_WARP0 + NUM_EPI_WARPS) * 32;
constexpr int MAX_STAGES = 16;
// TF32 tiles: columns of the accumulator one epilogue thread sums in registers
// (half of BLOCK_N <= 128), and the K elements one TMEM chunk accumulates.
constexpr int TF32_MAX_COLS = 64;
#ifndef KF_TF32_PROMOTE_K
#define KF_TF32_PROMOTE_K 128
#endif
constexpr int TF32_PROMOTE_K = KF_TF32_PROMOTE_K;
constexpr int MIN_SMEM_PER_CTA = 120 * 1024;  // > half an SM: one CTA per SM
constexpr uint64_t DRAIN_LIMIT_NS = 100000000ull;
// Stream-K workspace layout: [tile arrival counters | 2 partial tiles per CTA];
// SK_MAX_TILES and SK_COUNTER_BYTES live in kf_internal.h.

struct TcParams {
  int M, N, K;  // as the kernel sees them (after an optional A/B swap)
  int bn, bk, stages, group_m;
  int a_mn, b_mn;
  int tiles_m, tiles_n, kb_per_tile;
  long long total_iters;
  // Schedule: tiles [0, dp_tiles) go whole to unit t % units. Then either
  // (split tail) the remaining tiles are cut into two half-width tiles each,
  // dealt out the same way -- the last partial wave takes half as long, with
  // no K split and no fix-up -- or (stream-K) the k-block iterations
  // [sk_base, sk_base + sk_iters) of the remaining tiles are split evenly over
  // the units with a fixed-order fix-up.
  long long dp_tiles, sk_base, sk_iters;
  int tail_halves;  // half-width tiles after the whole ones (split tail)
  int stream_k;     // sk_iters > 0
  // k-blocks per TMEM accumulation chunk (0: a segment is one chunk). The
  // epilogue sums the chunks in fp32 registers: kind::tf32 accumulation over
  // thousands of k loses bits (3xTF32 at K = 4096 measured 1.0e-5 relative
  // error in one chunk, 5.7e-7 in chunks of 192).
  int promote_kb;
  int tf32_kp;  // TF32: elements between a split operand's small and big segments
  uint32_t idesc_half;
  void* c;
  long long sc_r, sc_c;
  const void* bias;
  int bias_on_rows;
  float* partials;
  int* counters;
  // Peer copies of C, written with the same offsets (all-gather epilogue).
  void* peers[KF_MAX_PEERS];
  int n_peers;
  // Whole 64-column chunks go through the shared-memory stage: 1 = written
  // out by the warp's stores, 2 = by TMA tensor stores (one per destination).
  int peer_stage;
  int* status;
  uint32_t idesc;
  uint32_t a_stage_bytes, b_stage_bytes;  // per CTA
  uint32_t tmem_cols;
};

struct Segment {
  int tile;
  int kb0, kb1;
  int half;  // -1: a whole tile; 0 / 1: the first / second half-width tile of it
};

struct Cursor {
  long long dp_next;          // next whole tile
  long long next, end, begin;  // stream-K iteration range [begin, end)
};

// First k-block iteration of a unit's stream-K range.
__device__ __forceinline__ long long sk_begin_of(const TcParams& p, long long unit, long long units) {
  return p.sk_base + (p.sk_iters * unit) / units;
}

// `unit` is the CTA (CG = 1) or the CTA pair (CG = 2); `units` their number.
__device__ __forceinline__ void cursor_init(const TcParams& p, Cursor& c, int unit, int units) {
  c.dp_next = unit;
  c.begin = sk_begin_of(p, unit, units);
  c.end = sk_begin_of(p, unit + 1, units);
  c.next = c.begin;
}

__device__ __forceinline__ bool cursor_next(const TcParams& p, Cursor& c, Segment& s, int units) {
  if (c.dp_next < p.dp_tiles) {
    s.tile = static_cast<int>(c.dp_next);
    s.kb0 = 0;
    s.kb1 = p.kb_per_tile;
    s.half = -1;
    c.dp_next += units;
    return true;
  }
  if (c.dp_next < p.dp_tiles + p.tail_halves) {
    const long long j = c.dp_next - p.dp_tiles;
    s.tile = static_cast<int>(p.dp_tiles + j / 2);
    s.half = static_cast<int>(j & 1);
    s.kb0 = 0;
    s.kb1 = p.kb_per_tile;
    c.dp_next += units;
    return true;
  }
  s.half = -1;
  if (c.next >= c.end) return false;
  const long long tile = c.next / p.kb_per_tile;
  const long long tile_start = tile * p.kb_per_tile;
  long long stop = c.end - tile_start;
  if (stop > p.kb_per_tile) stop = p.kb_per_tile;
  s.tile = static_cast<int>(tile);
  s.kb0 = static_cast<int>(c.next - tile_start);
  s.kb1 = static_cast<int>(stop);
  c.next = tile_start + stop;
  return true;
}

// Grouped raster: GROUP_M consecutive M tiles share each N column, so the CTAs
// resident at one time touch a compact block of C and its A/B panels stay in L2.
__device__ __forceinline__ void tile_coords(const TcParams& p, int tile, int& m_blk, int& n_blk) {
  const int per_group = p.group_m * p.tiles_n;
  const int gid = tile / per_group;
  const int first_m = gid * p.group_m;
  int rows = p.tiles_m - first_m;
  if (rows > p.group_m) rows = p.group_m;
  const int r = tile - gid * per_group;
  m_blk = first_m + r % rows;
  n_blk = r / rows;
}

// Stream-K: the CTA whose iteration range contains iteration x.
__device__ __forceinline__ long long owner_of(long long x, long long total, long long grid) {
  return ((x + 1) * grid + total - 1) / total - 1;
}

__device__ __forceinline__ void epi_bar_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(NUM_EPI_THREADS) : "memory");
}

// Epilogue for 16 accumulator columns of one row: bias, activation, rounding, store.
// Two fp32 values rounded to one packed pair of 16-bit values.
template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  uint32_t out;
  if constexpr (DType<T>::code == KF_BF16) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    memcpy(&out, &v, 4);
  } else {
    const __half2 v = __floats2half2_rn(lo, hi);
    memcpy(&out, &v, 4);
  }
  return out;
}

// Bias for 16 consecutive columns starting at col0 (zero past N).
template <typename T>
__device__ __forceinline__ void load_bias16(const T* bias, int col0, int n, float (&b)[16]) {
  if (col0 + 16 <= n && (reinterpret_cast<uintptr_t>(bias + col0) & 15u) == 0) {
    constexpr int PER_VEC = 16 / static_cast<int>(sizeof(T));
    const uint4* src = reinterpret_cast<const uint4*>(bias + col0);
#pragma unroll
    for (int v = 0; v < 16 / PER_VEC; ++v) {
      const uint4 q = __ldg(src + v);
      const T* e = reinterpret_cast<const T*>(&q);
#pragma unroll
      for (int j = 0; j < PER_VEC; ++j) b[v * PER_VEC + j] = to_f32(e[j]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) b[j] = col0 + j < n ? to_f32(__ldg(bias + col0 + j)) : 0.0f;
  }
}

// Bias and activation for one lane's 16 accumulators (row `row`, columns
// col0 .. col0 + 15).
template <typename T, int EPI>
__device__ __forceinline__ void epilogue16(const TcParams& p, int row, int col0, const float* acc,
                                           float (&v)[16]) {
  const T* bias = static_cast<const T*>(p.bias);
  if constexpr (EPI != KF_EPI_NONE) {
    float b[16];
    if (p.bias_on_rows) {
      const float rb = to_f32(bias[row]);
#pragma unroll
      for (int j = 0; j < 16; ++j) b[j] = rb;
    } else {
      load_bias16<T>(bias, col0, p.N, b);
    }
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
      const float2 r = apply_epilogue2<EPI>(make_float2(acc[j], acc[j + 1]), make_float2(b[j], b[j + 1]));
      v[j] = r.x;
      v[j + 1] = r.y;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = acc[j];
  }
}

template <typename T, int EPI, bool PEERS>
__device__ __forceinline__ void store_chunk(const TcParams& p, int row, int col0, const float* acc) {
  if (row >= p.M) return;
  float v[16];
  epilogue16<T, EPI>(p, row, col0, acc, v);
  const long long off = static_cast<long long>(row) * p.sc_r + static_cast<long long>(col0) * p.sc_c;
  T* out = static_cast<T*>(p.c) + off;
  const bool vec_ok = p.sc_c == 1 && col0 + 16 <= p.N && (reinterpret_cast<uintptr_t>(out) & 15u) == 0;
  if constexpr (sizeof(T) == 4) {
    // fp32 output (no peers on this path): 64 bytes as four 16-byte stores
    if (vec_ok) {
      float4* dst = reinterpret_cast<float4*>(out);
#pragma unroll
      for (int q = 0; q < 4; ++q) dst[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (col0 + j < p.N) out[static_cast<long long>(j) * p.sc_c] = v[j];
    }
    return;
  }
  if (vec_ok) {
    uint32_t packed[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) packed[j] = pack2<T>(v[2 * j], v[2 * j + 1]);
    const uint4 q0 = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    const uint4 q1 = make_uint4(packed[4], packed[5], packed[6], packed[7]);
    uint4* dst = reinterpret_cast<uint4*>(out);
    dst[0] = q0;
    dst[1] = q1;
    // The same 32 bytes into every peer's copy (NVLink stores; the peers'
    // buffers share this layout, so their 16-byte alignment matches).
    if constexpr (PEERS) {
      for (int i = 0; i < p.n_peers; ++i) {
        uint4* pd = reinterpret_cast<uint4*>(static_cast<T*>(p.peers[i]) + off);
        pd[0] = q0;
        pd[1] = q1;
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (col0 + j < p.N) {
        const T val = from_f32<T>(v[j]);
        out[static_cast<long long>(j) * p.sc_c] = val;
        if constexpr (PEERS) {
          for (int i = 0; i < p.n_peers; ++i)
            (static_cast<T*>(p.peers[i]) + off)[static_cast<long long>(j) * p.sc_c] = val;
        }
      }
    }
  }
}

// All-gather epilogue for 64 columns of a warp's 32 rows. Stores straight
// from the TMEM lane layout (one row per lane) would send each row's bytes as
// a separate 16-byte write over NVLink. Instead the warp stages its 32 x 64
// block in shared memory (16-byte segments XOR-swizzled by row, so both the
// row-per-lane writes and the segment-per-lane reads are conflict-free) and
// reads it back so that every store instruction covers 4 rows x 128
// contiguous bytes, sent to this GPU's C and to every peer's copy.
// Requires: 2-byte T, unit column stride, 16-byte aligned row starts in C and
// in every peer copy, and col0 + 64 <= N (the caller checks).
// Stage 16 columns (segments 2q and 2q + 1 of the lane's row).
template <typename T, int EPI>
__device__ __forceinline__ void stage16(const TcParams& p, int row, int lane, int col0, int q,
                                        const uint32_t (&r)[16], uint4* stage) {
  static_assert(sizeof(T) == 2, "the staged epilogue packs 2-byte elements");
  float v[16];
  epilogue16<T, EPI>(p, row, col0 + 16 * q, reinterpret_cast<const float*>(r), v);
  uint32_t packed[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) packed[j] = pack2<T>(v[2 * j], v[2 * j + 1]);
  stage[lane * 8 + ((2 * q) ^ (lane & 7))] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
  stage[lane * 8 + ((2 * q + 1) ^ (lane & 7))] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
}

// Write the staged 32 x 64 block (see stage16) to C and every peer copy.
template <typename T>
__device__ __forceinline__ void flush_stage64(const TcParams& p, int row_base, int lane, int col0,
                                              const uint4* stage) {
  __syncwarp();
  const int seg = lane & 7;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r_local = 4 * i + (lane >> 3);
    const uint4 val = stage[r_local * 8 + (seg ^ (r_local & 7))];
    const int grow = row_base + r_local;
    if (grow < p.M) {
      const long long off = static_cast<long long>(grow) * p.sc_r + col0 + 8 * seg;
      *reinterpret_cast<uint4*>(static_cast<T*>(p.c) + off) = val;
      // Each CTA starts with a different peer, so that every GPU receives
      // from all the others at once rather than all of them in turn.
      int k = static_cast<int>(blockIdx.x % static_cast<unsigned>(p.n_peers));
      for (int kk = 0; kk < p.n_peers; ++kk) {
        *reinterpret_cast<uint4*>(static_cast<T*>(p.peers[k]) + off) = val;
        if (++k == p.n_peers) k = 0;
      }
    }
  }
  __syncwarp();  // the stage is free for the next chunk
}

// Tensor maps of C and of the peers' copies for the TMA-store epilogue
// (box: 64 columns x 32 rows, 128-byte swizzle); the plain GEMM takes a
// 4-byte placeholder instead.
template <bool PEERS>
struct OutMaps {
  CUtensorMap m[KF_MAX_PEERS + 1];
};
template <>
struct OutMaps<false> {
  int unused;
};

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t smem_src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_src), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// The staged block has been read out of shared memory by every earlier store.
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Every earlier bulk store has completed (its writes are performed).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// PEERS: the all-gathering variant (every output tile also stored into the
// peers' copies of C); the plain GEMM is compiled without any of that code.
template <typename T, int EPI, int CG, bool PEERS>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tm_a,
                   const __grid_constant__ CUtensorMap tm_b,
                   const __grid_constant__ CUtensorMap tm_b_half, const TcParams p,
                   const __grid_constant__ OutMaps<PEERS> out_maps) {
  extern __shared__ uint8_t smem_raw[];
  // Elements in one 128-byte swizzle row (64 16-bit, 32 fp32), and per MMA K
  // step (32 bytes: K = 16 for kind::f16, 8 for kind::tf32).
  constexpr int ATOM = 128 / static_cast<int>(sizeof(T));
  constexpr bool TF32 = sizeof(T) == 4;
  static_assert(!(TF32 && PEERS), "the all-gather epilogue is compiled for 16-bit outputs");
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int S = p.stages;
  uint8_t* a_ring = smem;
  uint8_t* b_ring = smem + static_cast<size_t>(S) * p.a_stage_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(b_ring + static_cast<size_t>(S) * p.b_stage_bytes);
  // bars: full[S] | empty[S] | tmem_full[2] | tmem_empty[2] | drain
  uint32_t* misc = reinterpret_cast<uint32_t*>(bars + 2 * S + 5);
  // misc[0] TMEM base address, misc[1] abort flag, misc[2] "last contributor" flag
  volatile int* abort_flag = reinterpret_cast<volatile int*>(&misc[1]);
  volatile uint32_t* last_flag = &misc[2];
  // The all-gather epilogue's per-warp stages (allocated only when peer_stage).
  uint4* peer_stage = reinterpret_cast<uint4*>((reinterpret_cast<uintptr_t>(misc + 4) + 1023) &
                                               ~static_cast<uintptr_t>(1023));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t full0 = smem_u32(bars);
  const uint32_t empty0 = smem_u32(bars + S);
  const uint32_t tfull0 = smem_u32(bars + 2 * S);
  const uint32_t tempty0 = smem_u32(bars + 2 * S + 2);
  const uint32_t drain_bar = smem_u32(bars + 2 * S + 4);
  const uint32_t crank = CG == 2 ? cluster_ctarank() : 0u;
  const bool leader = crank == 0;
  const int unit = static_cast<int>(blockIdx.x) / CG;
  const int units = static_cast<int>(gridDim.x) / CG;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull0 + 8 * a, 1);
      // one arrival per epilogue warp of every CTA of the MMA group
      mbar_init(tempty0 + 8 * a, NUM_EPI_WARPS * CG);
    }
    mbar_init(drain_bar, 1);
    misc[1] = 0;
    misc[2] = 0;
    mbar_init_fence();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
    if (p.tail_halves) tma_prefetch_desc(&tm_b_half);
  }
  if (warp == 1) {
    if constexpr (CG == 2) {
      tmem_alloc_pair(smem_u32(&misc[0]), p.tmem_cols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(smem_u32(&misc[0]), p.tmem_cols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (CG == 2) {
    cluster_sync_all();  // the peer's TMA may target the leader's barriers from here on
  } else {
    __syncthreads();
  }
  tc_fence_after();
  const uint32_t tmem_base = misc[0];

  Cursor cur;
  cursor_init(p, cur, unit, units);
  Segment seg;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      long long issued = 0;
      bool ok = true;
      while (ok && cursor_next(p, cur, seg, units)) {
        int m_blk, n_blk;
        tile_coords(p, seg.tile, m_blk, n_blk);
        // A half-width tile stages half the B rows, through the half-height map.
        const bool half = seg.half >= 0;
        const int seg_bn = half ? p.bn / 2 : p.bn;
        const int b_rows = seg_bn / CG;  // B rows this CTA stages
        const CUtensorMap* map_b = half ? &tm_b_half : &tm_b;
        // TF32: a stage holds both parts of the k-block, small then big
        // (segments 0 and 1 of the split operands, kp elements apart).
        constexpr int PARTS = TF32 ? 2 : 1;
        const uint32_t tx_bytes =
            (p.a_stage_bytes + static_cast<uint32_t>(PARTS * b_rows * p.bk * static_cast<int>(sizeof(T)))) * CG;
        const int m0 = m_blk * (BM * CG) + BM * static_cast<int>(crank);
        const int n0 = n_blk * p.bn + (half ? seg.half * seg_bn : 0) + b_rows * static_cast<int>(crank);
        for (int kb = seg.kb0; kb < seg.kb1; ++kb) {
          if (!mbar_wait(empty0 + 8 * stage, phase ^ 1u, abort_flag, p.status, SITE_TMA_EMPTY)) {
            ok = false;
            break;
          }
          const uint32_t fb = full0 + 8 * stage;
          const int k0 = kb * p.bk;
          const uint32_t a_dst = smem_u32(a_ring + static_cast<size_t>(stage) * p.a_stage_bytes);
          const uint32_t b_dst = smem_u32(b_ring + static_cast<size_t>(stage) * p.b_stage_bytes);
          if constexpr (CG == 2) {
            if (leader) mbar_arrive_expect_tx(fb, tx_bytes);
          } else {
            mbar_arrive_expect_tx(fb, tx_bytes);
          }
          // both CTAs of a pair count on the leader's barrier
          const uint32_t lb = CG == 2 ? mapa_shared(fb, 0) : fb;
#pragma unroll
          for (int part = 0; part < PARTS; ++part) {
            const uint32_t a_p = a_dst + part * (p.a_stage_bytes / PARTS);
            const uint32_t b_p = b_dst + part * (p.b_stage_bytes / PARTS);
            const int kx = k0 + part * p.tf32_kp;
            if constexpr (CG == 2) {
              if (!p.a_mn) {
                for (int j = 0; j < p.bk / ATOM; ++j)
                  tma_load_2d_pair(a_p + j * (BM * 128), &tm_a, lb, kx + ATOM * j, m0);
              } else {
                for (int i = 0; i < BM / ATOM; ++i)
                  tma_load_2d_pair(a_p + i * (p.bk * 128), &tm_a, lb, m0 + ATOM * i, kx);
              }
              if (!p.b_mn) {
                for (int j = 0; j < p.bk / ATOM; ++j)
                  tma_load_2d_pair(b_p + j * (b_rows * 128), map_b, lb, kx + ATOM * j, n0);
              } else {
                for (int i = 0; i < b_rows / ATOM; ++i)
                  tma_load_2d_pair(b_p + i * (p.bk * 128), map_b, lb, n0 + ATOM * i, kx);
              }
            } else {
              if (!p.a_mn) {
                for (int j = 0; j < p.bk / ATOM; ++j)
                  tma_load_2d(a_p + j * (BM * 128), &tm_a, lb, kx + ATOM * j, m0);
              } else {
                for (int i = 0; i < BM / ATOM; ++i)
                  tma_load_2d(a_p + i * (p.bk * 128), &tm_a, lb, m0 + ATOM * i, kx);
              }
              if (!p.b_mn) {
                for (int j = 0; j < p.bk / ATOM; ++j)
                  tma_load_2d(b_p + j * (b_rows * 128), map_b, lb, kx + ATOM * j, n0);
              } else {
                for (int i = 0; i < b_rows / ATOM; ++i)
                  tma_load_2d(b_p + i * (p.bk * 128), map_b, lb, n0 + ATOM * i, kx);
              }
            }
          }
          ++issued;
          if (++stage == static_cast<uint32_t>(S)) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && leader) {
        // Aborting: let every bulk copy already issued land before the CTA's
        // shared memory goes away. (A pair's copies all count on the leader's
        // barriers; the follower is held by the final cluster barrier.)
        for (int s = 0; s < S && s < issued; ++s) {
          const long long armed = (issued - s + S - 1) / S;
          mbar_wait(full0 + 8 * s, static_cast<uint32_t>((armed - 1) & 1), nullptr, p.status,
                    SITE_DRAIN, DRAIN_LIMIT_NS);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && leader) {
      uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
      bool ok = true;
      // Start-address steps in 16-byte units. K-major operands: an MMA's K
      // slice (16 16-bit or 8 fp32 elements) is 32 bytes inside a 128-byte
      // swizzle row, and the next K atom starts `rows * 128` bytes on.
      // MN-major operands (16-bit only): a K=16 slice is 16 K-rows of 128
      // bytes, and one 64-deep atom is 4 slices.
      const uint32_t a_k_step = p.a_mn ? 2048 / 16 : 32 / 16;
      const uint32_t b_k_step = p.b_mn ? 2048 / 16 : 32 / 16;
      const uint32_t a_atom_step = p.a_mn ? 4 * 2048 / 16 : (BM * 128) / 16;
      const uint32_t a_lbo = p.a_mn ? static_cast<uint32_t>(p.bk * 128) : 16u;
      const uint32_t b_lbo = p.b_mn ? static_cast<uint32_t>(p.bk * 128) : 16u;
      while (ok && cursor_next(p, cur, seg, units)) {
        // A segment's k-blocks accumulate in TMEM as one chunk, or (promote_kb
        // > 0) as chunks of promote_kb k-blocks, each into the next TMEM buffer,
        // summed by the epilogue in fp32 registers.
        for (int c0 = seg.kb0, c1; ok && c0 < seg.kb1; c0 = c1) {
          c1 = p.promote_kb > 0 && seg.kb1 - c0 > p.promote_kb ? c0 + p.promote_kb : seg.kb1;
          if (!mbar_wait(tempty0 + 8 * acc, acc_phase ^ 1u, abort_flag, p.status,
                         SITE_MMA_TMEM_EMPTY)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // A half-width tile: half the B rows per K atom and an N/2 instruction.
          const int b_rows = (seg.half >= 0 ? p.bn / 2 : p.bn) / CG;
          const uint32_t b_atom_step =
              p.b_mn ? 4 * 2048 / 16 : static_cast<uint32_t>(b_rows * 128) / 16;
          const uint32_t idesc = seg.half >= 0 ? p.idesc_half : p.idesc;
          const uint32_t d_tmem = tmem_base + acc * static_cast<uint32_t>(p.bn);
          for (int kb = c0; kb < c1; ++kb) {
            if (!mbar_wait(full0 + 8 * stage, phase, abort_flag, p.status, SITE_MMA_FULL)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_base = smem_u32(a_ring + static_cast<size_t>(stage) * p.a_stage_bytes);
            const uint32_t b_base = smem_u32(b_ring + static_cast<size_t>(stage) * p.b_stage_bytes);
            const uint64_t a_desc0 = smem_desc_sw128(a_base, a_lbo, 1024);
            const uint64_t b_desc0 = smem_desc_sw128(b_base, b_lbo, 1024);
            // The descriptors of one k-block differ only in their start address
            // (bits 0-13, 16-byte units): step by constants, issue unrolled.
            for (int atom = 0; atom < p.bk / ATOM; ++atom) {
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {
                const uint64_t a_desc = a_desc0 + static_cast<uint64_t>(atom * a_atom_step + kk * a_k_step);
                const uint64_t b_desc = b_desc0 + static_cast<uint64_t>(atom * b_atom_step + kk * b_k_step);
                const uint32_t accumulate = (kb > c0 || atom > 0 || kk > 0) ? 1u : 0u;
                if constexpr (TF32) {
                  // 3xTF32 on the stage's two parts: small x big, big x small,
                  // then big x big (the big halves sit half a stage on)
                  const uint64_t a_big = a_desc + (p.a_stage_bytes / 2) / 16;
                  const uint64_t b_big = b_desc + (p.b_stage_bytes / 2) / 16;
                  if constexpr (CG == 2) {
                    tc_mma_tf32_pair(d_tmem, a_desc, b_big, idesc, accumulate);
                    tc_mma_tf32_pair(d_tmem, a_big, b_desc, idesc, 1u);
                    tc_mma_tf32_pair(d_tmem, a_big, b_big, idesc, 1u);
                  } else {
                    tc_mma_tf32(d_tmem, a_desc, b_big, idesc, accumulate);
                    tc_mma_tf32(d_tmem, a_big, b_desc, idesc, 1u);
                    tc_mma_tf32(d_tmem, a_big, b_big, idesc, 1u);
                  }
                } else if constexpr (CG == 2) {
                  tc_mma_f16_pair(d_tmem, a_desc, b_desc, idesc, accumulate);
                } else {
                  tc_mma_f16(d_tmem, a_desc, b_desc, idesc, accumulate);
                }
              }
            }
            // ring slot reusable (in every CTA of the group) once these MMAs finish
            if constexpr (CG == 2) {
              tc_commit_pair_to(empty0 + 8 * stage, 0x3);
            } else {
              tc_commit(empty0 + 8 * stage);
            }
            if (++stage == static_cast<uint32_t>(S)) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (!ok) break;
          // accumulator complete: wake the epilogue of every CTA of the group
          if constexpr (CG == 2) {
            tc_commit_pair_to(tfull0 + 8 * acc, 0x3);
          } else {
            tc_commit(tfull0 + 8 * acc);
          }
          if (++acc == 2) {
            acc = 0;
            acc_phase ^= 1u;
          }
        }
      }
      // Every MMA issued must complete before TMEM is released.
      if constexpr (CG == 2) {
        tc_commit_pair(drain_bar);
      } else {
        tc_commit(drain_bar);
      }
      mbar_wait(drain_bar, 0, nullptr, p.status, SITE_DRAIN, DRAIN_LIMIT_NS);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;  // the TMEM lane quadrant this warp may read
    const int row_in_tile = quad * 32 + lane;
    const int ethread = threadIdx.x - EPI_WARP0 * 32;
    // Two warps share each quadrant: the first takes the first half of the
    // tile's 16-column chunks, the second the rest.
    const int half = (warp - EPI_WARP0) / 4;
    // The MMA leader's tmem_empty barriers (this CTA's own when CG = 1).
    const uint32_t tempty_leader = CG == 2 ? mapa_shared(tempty0, 0) : tempty0;
    uint32_t acc = 0, acc_phase = 0;
    while (cursor_next(p, cur, seg, units)) {
      if constexpr (TF32) {
        // TF32 tiles (BLOCK_N <= 128: at most 64 columns per thread): the
        // segment's TMEM chunks are summed into fp32 registers, then stored
        // (a whole tile) or fixed up (stream-K) from the registers.
        int m_blk, n_blk;
        tile_coords(p, seg.tile, m_blk, n_blk);
        const int seg_bn = seg.half >= 0 ? p.bn / 2 : p.bn;
        const int chunk_split = (seg_bn / 16 + 1) / 2;
        const int c_begin = half == 0 ? 0 : chunk_split * 16;
        const int c_end = half == 0 ? chunk_split * 16 : seg_bn;
        const int row = m_blk * (BM * CG) + BM * static_cast<int>(crank) + row_in_tile;
        const int col_base = n_blk * p.bn + (seg.half >= 0 ? seg.half * seg_bn : 0);
        float sums[TF32_MAX_COLS];
#pragma unroll
        for (int j = 0; j < TF32_MAX_COLS; ++j) sums[j] = 0.0f;
        bool ok = true;
        for (int c0 = seg.kb0, c1; c0 < seg.kb1; c0 = c1) {
          c1 = p.promote_kb > 0 && seg.kb1 - c0 > p.promote_kb ? c0 + p.promote_kb : seg.kb1;
          if (!mbar_wait(tfull0 + 8 * acc, acc_phase, abort_flag, p.status, SITE_EPI_TMEM_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t t_acc =
              tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * static_cast<uint32_t>(p.bn);
#pragma unroll
          for (int g = 0; g < TF32_MAX_COLS / 16; g += 2) {
            uint32_t r0[16], r1[16];
            // warp-uniform: c_begin and c_end depend on the warp only
            const bool on0 = c_begin + 16 * g < c_end, on1 = c_begin + 16 * (g + 1) < c_end;
            __syncwarp();
            if (on0) tmem_ld_16(t_acc + c_begin + 16 * g, r0);
            if (on1) tmem_ld_16(t_acc + c_begin + 16 * (g + 1), r1);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              if (on0) sums[16 * g + j] += __uint_as_float(r0[j]);
              if (on1) sums[16 * (g + 1) + j] += __uint_as_float(r1[j]);
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if constexpr (CG == 2) {
              mbar_arrive_cluster(tempty_leader + 8 * acc);
            } else {
              mbar_arrive(tempty0 + 8 * acc);
            }
          }
          if (++acc == 2) {
            acc = 0;
            acc_phase ^= 1u;
          }
        }
        if (!ok) break;
        if (seg.kb0 == 0 && seg.kb1 == p.kb_per_tile) {
#pragma unroll
          for (int g = 0; g < TF32_MAX_COLS / 16; ++g)
            if (c_begin + 16 * g < c_end) store_chunk<T, EPI, false>(p, row, col_base + c_begin + 16 * g, sums + 16 * g);
          continue;
        }
{
          // Stream-K fix-up from the registers, as for the 16-bit tiles below:
          // partials in [16-column chunk][row][16] slots, the last contributor
          // sums them in contributor order.
          const long long grid = units;
          const long long t_start = static_cast<long long>(seg.tile) * p.kb_per_tile;
          const long long rel = t_start - p.sk_base;
          const long long c_first = owner_of(rel, p.sk_iters, grid);
          const long long c_last = owner_of(rel + p.kb_per_tile - 1, p.sk_iters, grid);
          const long long me = unit;
          const size_t slot_elems = static_cast<size_t>(p.bn) * BM;
          const long long my_slot = 2 * (me * CG + crank) + (cur.begin >= t_start ? 0 : 1);
          float* mine = p.partials + static_cast<size_t>(my_slot) * slot_elems;
          int* counter = p.counters + static_cast<size_t>(seg.tile) * CG + crank;
#pragma unroll
          for (int g = 0; g < TF32_MAX_COLS / 16; ++g) {
            const int c = c_begin + 16 * g;
            if (c >= c_end) continue;
            float4* dst = reinterpret_cast<float4*>(mine + (static_cast<size_t>(c / 16) * BM + row_in_tile) * 16);
#pragma unroll
            for (int q = 0; q < 4; ++q)
              __stcg(dst + q, make_float4(sums[16 * g + 4 * q], sums[16 * g + 4 * q + 1], sums[16 * g + 4 * q + 2],
                                          sums[16 * g + 4 * q + 3]));
          }
          __threadfence();
          epi_bar_sync();
          if (ethread == 0) {
            const int arrived = atomicAdd(counter, 1);
            *last_flag = (arrived == static_cast<int>(c_last - c_first)) ? 1u : 0u;
          }
          epi_bar_sync();
          if (*last_flag) {
            __threadfence();
#pragma unroll
            for (int g = 0; g < TF32_MAX_COLS / 16; ++g) {
              const int c = c_begin + 16 * g;
              if (c >= c_end) continue;
              float sum[16];
#pragma unroll
              for (int j = 0; j < 16; ++j) sum[j] = 0.0f;
              for (long long cc = c_first; cc <= c_last; ++cc) {
                if (cc == me) {
#pragma unroll
                  for (int j = 0; j < 16; ++j) sum[j] += sums[16 * g + j];
                  continue;
                }
                const long long cc_begin = sk_begin_of(p, cc, grid);
                const long long slot = 2 * (cc * CG + crank) + (cc_begin >= t_start ? 0 : 1);
                const float4* part = reinterpret_cast<const float4*>(
                    p.partials + static_cast<size_t>(slot) * slot_elems + (static_cast<size_t>(c / 16) * BM + row_in_tile) * 16);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  const float4 v = __ldcg(part + q);
                  sum[4 * q] += v.x;
                  sum[4 * q + 1] += v.y;
                  sum[4 * q + 2] += v.z;
                  sum[4 * q + 3] += v.w;
                }
              }
              store_chunk<T, EPI, false>(p, row, col_base + c, sum);
            }
            if (ethread == 0) *counter = 0;  // leave the workspace clean
          }
          epi_bar_sync();
        }
        continue;
      }
      if (!mbar_wait(tfull0 + 8 * acc, acc_phase, abort_flag, p.status, SITE_EPI_TMEM_FULL)) break;
      tc_fence_after();
      int m_blk, n_blk;
      tile_coords(p, seg.tile, m_blk, n_blk);
      const int seg_bn = seg.half >= 0 ? p.bn / 2 : p.bn;
      const int chunks = seg_bn / 16;
      const int chunk_split = (chunks + 1) / 2;
      const int c_begin = half == 0 ? 0 : chunk_split * 16;
      const int c_end = half == 0 ? chunk_split * 16 : seg_bn;
      const int row = m_blk * (BM * CG) + BM * static_cast<int>(crank) + row_in_tile;
      const int col_base = n_blk * p.bn + (seg.half >= 0 ? seg.half * seg_bn : 0);
      const uint32_t t_acc =
          tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * static_cast<uint32_t>(p.bn);
      const bool whole_tile = seg.kb0 == 0 && seg.kb1 == p.kb_per_tile;
      if (whole_tile) {
        int c = c_begin;
        if constexpr (PEERS) {
          if (p.peer_stage) {
            uint4* stage = peer_stage + (warp - EPI_WARP0) * (32 * 8);
            const int row_base = row - lane;
            const bool tma = p.peer_stage == 2;
            // TMA stores clip at the tensor's edge, so a ragged last chunk
            // still goes through the stage; thread stores need whole chunks.
            const int n_limit = tma ? p.N : p.N - 63;
            for (; c + 64 <= c_end && col_base + c < n_limit; c += 64) {
              if (tma) {
                if (lane == 0) bulk_wait_read_all();  // the previous chunk has left the stage
                __syncwarp();
              }
  #pragma unroll
              for (int q = 0; q < 4; q += 2) {  // two 16-column TMEM loads in flight per wait
                uint32_t r0[16], r1[16];
                __syncwarp();
                tmem_ld_16(t_acc + c + 16 * q, r0);
                tmem_ld_16(t_acc + c + 16 * q + 16, r1);
                tmem_ld_wait();
                stage16<T, EPI>(p, row, lane, col_base + c, q, r0, stage);
                stage16<T, EPI>(p, row, lane, col_base + c, q + 1, r1, stage);
              }
              if (tma) {
                fence_async_shared();  // the stage writes are visible to the TMA unit
                __syncwarp();
                if (lane == 0 && row_base < p.M) {  // (no store starts past the last row)
                  const uint32_t src = smem_u32(stage);
                  tma_store_2d(&out_maps.m[0], src, col_base + c, row_base);
                  // peers from a different one per CTA (see flush_stage64)
                  int k = static_cast<int>(blockIdx.x % static_cast<unsigned>(p.n_peers));
                  for (int kk = 0; kk < p.n_peers; ++kk) {
                    tma_store_2d(&out_maps.m[1 + k], src, col_base + c, row_base);
                    if (++k == p.n_peers) k = 0;
                  }
                  bulk_commit_group();
                }
              } else {
                flush_stage64<T>(p, row_base, lane, col_base + c, stage);
              }
            }
          }
        }
        // Two 16-column TMEM loads in flight per wait.
        for (; c < c_end; c += 32) {
          uint32_t r0[16], r1[16];
          const bool two = c + 16 < c_end;
          __syncwarp();  // tcgen05.ld is .sync.aligned
          tmem_ld_16(t_acc + c, r0);
          if (two) tmem_ld_16(t_acc + c + 16, r1);
          tmem_ld_wait();
          store_chunk<T, EPI, PEERS>(p, row, col_base + c, reinterpret_cast<const float*>(r0));
          if (two) store_chunk<T, EPI, PEERS>(p, row, col_base + c + 16, reinterpret_cast<const float*>(r1));
        }
      } else {
        // Stream-K fix-up for a tile shared between units. Each CTA fixes up
        // its own 128 rows: its own counter and its own partial slots (a
        // unit's first and last segment), so the two CTAs of a pair proceed
        // independently.
        const long long grid = units;
        const long long t_start = static_cast<long long>(seg.tile) * p.kb_per_tile;
        const long long rel = t_start - p.sk_base;
        const long long c_first = owner_of(rel, p.sk_iters, grid);
        const long long c_last = owner_of(rel + p.kb_per_tile - 1, p.sk_iters, grid);
        const long long me = unit;
        const size_t slot_elems = static_cast<size_t>(p.bn) * BM;
        const long long my_slot = 2 * (me * CG + crank) + (cur.begin >= t_start ? 0 : 1);
        float* mine = p.partials + static_cast<size_t>(my_slot) * slot_elems;
        int* counter = p.counters + static_cast<size_t>(seg.tile) * CG + crank;
        // Partial tiles are laid out [16-column chunk][row][16]: a lane's 16
        // columns are 64 contiguous bytes and a warp's stores cover 2 KB.
        for (int c = c_begin; c < c_end; c += 16) {
          uint32_t r[16];
          __syncwarp();
          tmem_ld_16(t_acc + c, r);
          tmem_ld_wait();
          float4* dst = reinterpret_cast<float4*>(mine + (static_cast<size_t>(c / 16) * BM + row_in_tile) * 16);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            __stcg(dst + q, make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                        __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3])));
        }
        __threadfence();
        epi_bar_sync();
        if (ethread == 0) {
          const int arrived = atomicAdd(counter, 1);
          *last_flag = (arrived == static_cast<int>(c_last - c_first)) ? 1u : 0u;
        }
        epi_bar_sync();
        if (*last_flag) {
          __threadfence();
          // The contributors' partials of a chunk are loaded FIX_BATCH at a
          // time, all loads in flight together (one L2 round trip per batch,
          // not per contributor), then summed in contributor order -- the
          // same fixed order, so the result stays deterministic.
          constexpr int FIX_BATCH = 2;
          for (int c = c_begin; c < c_end; c += 16) {
            uint32_t r[16];
            __syncwarp();
            tmem_ld_16(t_acc + c, r);
            float sum[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) sum[j] = 0.0f;
            for (long long cc0 = c_first; cc0 <= c_last; cc0 += FIX_BATCH) {
              float4 v[FIX_BATCH][4];
#pragma unroll
              for (int bi = 0; bi < FIX_BATCH; ++bi) {
                const long long cc = cc0 + bi;
                if (cc <= c_last && cc != me) {
                  const long long cc_begin = sk_begin_of(p, cc, grid);
                  const long long slot = 2 * (cc * CG + crank) + (cc_begin >= t_start ? 0 : 1);
                  const float4* part = reinterpret_cast<const float4*>(
                      p.partials + static_cast<size_t>(slot) * slot_elems +
                      (static_cast<size_t>(c / 16) * BM + row_in_tile) * 16);
#pragma unroll
                  for (int q = 0; q < 4; ++q) v[bi][q] = __ldcg(part + q);
                }
              }
              if (cc0 == c_first) tmem_ld_wait();
#pragma unroll
              for (int bi = 0; bi < FIX_BATCH; ++bi) {
                const long long cc = cc0 + bi;
                if (cc > c_last) break;
                if (cc == me) {
#pragma unroll
                  for (int j = 0; j < 16; ++j) sum[j] += __uint_as_float(r[j]);
                } else {
#pragma unroll
                  for (int q = 0; q < 4; ++q) {
                    sum[4 * q] += v[bi][q].x;
                    sum[4 * q + 1] += v[bi][q].y;
                    sum[4 * q + 2] += v[bi][q].z;
                    sum[4 * q + 3] += v[bi][q].w;
                  }
                }
              }
            }
            store_chunk<T, EPI, PEERS>(p, row, col_base + c, sum);
          }
          if (ethread == 0) *counter = 0;  // leave the workspace clean
        }
        epi_bar_sync();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (CG == 2) {
          mbar_arrive_cluster(tempty_leader + 8 * acc);
        } else {
          mbar_arrive(tempty0 + 8 * acc);
        }
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  // The TMA stores into peers' memory complete before the CTA (and its shared
  // memory) goes away. No system fence here: the peer barrier that follows on
  // the stream starts after this kernel completes and fences at system scope
  // before it signals (a fence.sc.sys per CTA measured +9 us on the tile GEMV).
  if (PEERS && warp >= EPI_WARP0) {
    if (p.peer_stage == 2 && lane == 0) bulk_wait_all();  // this warp's TMA stores are done
    __syncwarp();
  }
  tc_fence_before();
  __syncwarp();  // lanes 1-31 of warps 0 and 1 arrive here before their lane 0
  if constexpr (CG == 2) {
    cluster_sync_all();  // both CTAs done: no MMA, TMEM read or remote arrive in flight
  } else {
    __syncthreads();
  }
  if (warp == 1) {
    __syncwarp();  // tcgen05.dealloc is .sync.aligned: the whole warp, converged
    tc_fence_after();
    if constexpr (CG == 2) {
      tmem_dealloc_pair(tmem_base, p.tmem_cols);
    } else {
      tmem_dealloc(tmem_base, p.tmem_cols);
    }
  }
}

// ------------------------------------------------------------------- host side

uint32_t tmem_cols_for(int bn) {
  uint32_t need = static_cast<uint32_t>(2 * bn);
  uint32_t cols = 32;
  while (cols < need) cols <<= 1;
  return cols;
}

int elem_bytes(int dtype) { return dtype == KF_FP32 ? 4 : 2; }
// Bytes a ring stage holds per (row, k): TF32 stages carry both split parts.
int stage_elem_bytes(int dtype) { return dtype == KF_FP32 ? 8 : 2; }

// Shared memory of one CTA: A rows (128) and this CTA's B rows per stage.
int64_t smem_bytes_for(int bn, int bk, int stages, int cg, int elem, bool peer_stage = false) {
  const int64_t ring = static_cast<int64_t>(stages) * (BM + bn / cg) * bk * elem;
  return 1024 + ring + 8 * (2 * stages + 5) + 16 + (peer_stage ? GEMM_PEER_STAGE_SMEM : 0);
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* sym = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &sym, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(sym);
    }
  });
  return fn;
}

// A 2-D view [outer][inner] with `outer_stride` elements between rows; the box
// is `box_inner` x `box_outer` elements (box_inner x element size = 128 bytes
// for the swizzled operand tiles).
int encode_map(CUtensorMap* map, int dtype, const void* ptr, uint64_t inner, uint64_t outer,
               int64_t outer_stride, uint32_t box_inner, uint32_t box_outer) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return set_error(KF_ERR_LAUNCH, "cuTensorMapEncodeTiled unavailable");
  const int elem = elem_bytes(dtype);
  int64_t stride_bytes = outer_stride * elem;
  if (outer <= 1) stride_bytes = ((static_cast<int64_t>(inner) * elem + 15) / 16) * 16;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(stride_bytes)};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t elem_strides[2] = {1, 1};
  const CUtensorMapDataType t = dtype == KF_FP32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                : dtype == KF_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                   : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = enc(map, t, 2, const_cast<void*>(ptr), dims, strides, box, elem_strides,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    return set_error(KF_ERR_UNALIGNED,
                     "cuTensorMapEncodeTiled rejected the operand (error " + std::to_string(r) +
                         ", inner=" + std::to_string(inner) + ", outer=" + std::to_string(outer) +
                         ", stride_bytes=" + std::to_string(stride_bytes) + ")");
  }
  return KF_OK;
}

// The kernel's view of the problem after an optional swap of A and B.
struct View {
  const void* a;
  int64_t sa_r, sa_k;  // A'(r, k)
  const void* b;
  int64_t sb_k, sb_c;  // B'(k, c)
  int64_t sc_r, sc_c;  // C'(r, c)
  int64_t M, N;
  bool bias_on_rows;
};

View make_view(const GemmArgs& g, bool swap) {
  View v;
  if (!swap) {
    v = View{g.a, g.sa_m, g.sa_k, g.b, g.sb_k, g.sb_n, g.sc_m, g.sc_n, g.M, g.N, false};
  } else {
    // C^T = B^T A^T: A'(n, k) = B(k, n), B'(k, m) = A(m, k), C'(n, m) = C(m, n).
    v = View{g.b, g.sb_n, g.sb_k, g.a, g.sa_k, g.sa_m, g.sc_n, g.sc_m, g.N, g.M, true};
  }
  return v;
}

// Operand majorness for TMA: 0 = K-major, 1 = MN-major, -1 = not describable.
int operand_major(const void* ptr, int64_t s_mn, int64_t s_k, int64_t mn, int64_t k) {
  if ((reinterpret_cast<uintptr_t>(ptr) & 15u) != 0) return -1;
  if (k < 8) return -1;
  if (s_k == 1 && (mn == 1 || (s_mn % 8 == 0 && s_mn >= k))) return 0;
  if (s_mn == 1 && s_k % 8 == 0 && s_k >= mn) return 1;
  return -1;
}

template <typename T, int EPI>
void* kernel_ptr(int cg, bool peers) {
  if (peers)
    return cg == 2 ? reinterpret_cast<void*>(&tc_gemm_kernel<T, EPI, 2, true>)
                   : reinterpret_cast<void*>(&tc_gemm_kernel<T, EPI, 1, true>);
  return cg == 2 ? reinterpret_cast<void*>(&tc_gemm_kernel<T, EPI, 2, false>)
                 : reinterpret_cast<void*>(&tc_gemm_kernel<T, EPI, 1, false>);
}

void* pick_kernel(int dtype, int epi, int cg, bool peers) {
  if (dtype == KF_FP32) {  // TF32 split operands; never with peers (checked by the caller)
    switch (epi) {
      case KF_EPI_NONE: return cg == 2 ? reinterpret_cast<void*>(&tc_gemm_kernel<float, KF_EPI_NONE, 2, false>)
                                       : reinterpret_cast<void*>(&tc_gemm_kernel<float, KF_EPI_NONE, 1, false>);
      case KF_EPI_BIAS: return cg == 2 ? reinterpret_cast<void*>(&tc_gemm_kernel<float, KF_EPI_BIAS, 2, false>)
                                       : reinterpret_cast<void*>(&tc_gemm_kernel<float, KF_EPI_BIAS, 1, false>);
      case KF_EPI_BIAS_GELU_TANH:
        return cg == 2 ? reinterpret_cast<void*>(&tc_gemm_kernel<float, KF_EPI_BIAS_GELU_TANH, 2, false>)
                       : reinterpret_cast<void*>(&tc_gemm_kernel<float, KF_EPI_BIAS_GELU_TANH, 1, false>);
      default:
        return cg == 2 ? reinterpret_cast<void*>(&tc_gemm_kernel<float, KF_EPI_BIAS_GELU_ERF, 2, false>)
                       : reinterpret_cast<void*>(&tc_gemm_kernel<float, KF_EPI_BIAS_GELU_ERF, 1, false>);
    }
  }
  if (dtype == KF_FP16) {
    switch (epi) {
      case KF_EPI_NONE: return kernel_ptr<__half, KF_EPI_NONE>(cg, peers);
      case KF_EPI_BIAS: return kernel_ptr<__half, KF_EPI_BIAS>(cg, peers);
      case KF_EPI_BIAS_GELU_TANH: return kernel_ptr<__half, KF_EPI_BIAS_GELU_TANH>(cg, peers);
      default: return kernel_ptr<__half, KF_EPI_BIAS_GELU_ERF>(cg, peers);
    }
  }
  switch (epi) {
    case KF_EPI_NONE: return kernel_ptr<__nv_bfloat16, KF_EPI_NONE>(cg, peers);
    case KF_EPI_BIAS: return kernel_ptr<__nv_bfloat16, KF_EPI_BIAS>(cg, peers);
    case KF_EPI_BIAS_GELU_TANH: return kernel_ptr<__nv_bfloat16, KF_EPI_BIAS_GELU_TANH>(cg, peers);
    default: return kernel_ptr<__nv_bfloat16, KF_EPI_BIAS_GELU_ERF>(cg, peers);
  }
}

int cta_group_of(const kf_gemm_config& cfg) { return cfg.block_m == 2 * BM ? 2 : 1; }

int validate_config(const kf_gemm_config& cfg, int b_mn, int dtype, std::string* why) {
  if (cfg.block_m != BM && cfg.block_m != 2 * BM) {
    *why = "tcgen05 path supports BLOCK_M=128 (one SM) or 256 (an SM pair); got " +
           std::to_string(cfg.block_m);
    return KF_ERR_INVALID_CONFIG;
  }
  const int cg = cta_group_of(cfg);
  if (cfg.block_n < 16 || cfg.block_n > 256 || cfg.block_n % (16 * cg) != 0) {
    *why = "BLOCK_N must be a multiple of " + std::to_string(16 * cg) + " in [16, 256]; got " +
           std::to_string(cfg.block_n);
    return KF_ERR_INVALID_CONFIG;
  }
  if (b_mn == 1 && (cfg.block_n / cg) % 64 != 0) {
    *why = "an MN-major B operand needs each CTA's BLOCK_N share to be a multiple of 64";
    return KF_ERR_INVALID_CONFIG;
  }
  if (dtype == KF_FP32 && cfg.block_n > 2 * TF32_MAX_COLS) {
    *why = "TF32 tiles sum their accumulator chunks in registers: BLOCK_N must be at most " +
           std::to_string(2 * TF32_MAX_COLS) + "; got " + std::to_string(cfg.block_n);
    return KF_ERR_INVALID_CONFIG;
  }
  // One or two 128-byte swizzle atoms of K: 64 or 128 16-bit elements, 32 or
  // 64 fp32 (TF32) elements.
  const int atom = 128 / elem_bytes(dtype);
  if (cfg.block_k != atom && cfg.block_k != 2 * atom) {
    *why = "BLOCK_K must be " + std::to_string(atom) + " or " + std::to_string(2 * atom) +
           " (whole 128-byte swizzle atoms); got " + std::to_string(cfg.block_k);
    return KF_ERR_INVALID_CONFIG;
  }
  if (cfg.stages < 2 || cfg.stages > MAX_STAGES) {
    *why = "stages must be in [2, 16]; got " + std::to_string(cfg.stages);
    return KF_ERR_INVALID_CONFIG;
  }
  if (cfg.epi_store < 0 || cfg.epi_store > 2) {
    *why = "epi_store must be 0 (library choice), 1 (thread stores) or 2 (TMA stores)";
    return KF_ERR_INVALID_CONFIG;
  }
  if (cfg.cluster_n > 1 || (cg == 1 && cfg.cluster_m > 1) || (cg == 2 && cfg.cluster_m > 2)) {
    *why = "clusters beyond the SM pair of a BLOCK_M=256 tile are not implemented";
    return KF_ERR_INVALID_CONFIG;
  }
  if (cfg.stream_k < 0 || cfg.stream_k > 3) {
    *why = "stream_k must be 0 (library choice), 1 (all), 2 (off) or 3 (split tail)";
    return KF_ERR_INVALID_CONFIG;
  }
  if (cfg.group_m < 1) {
    *why = "GROUP_M must be positive";
    return KF_ERR_INVALID_CONFIG;
  }
  return KF_OK;
}

}  // namespace

bool tma_describable(const void* ptr, int64_t s_mn, int64_t s_k, int64_t mn, int64_t k) {
  return operand_major(ptr, s_mn, s_k, mn, k) >= 0;
}

bool tcgen05_operands_ok(const GemmArgs& g, std::string* why) {
  if (g.dtype == KF_FP32) {
    // fp32 runs as 3xTF32 on operands split into TF32 parts (tf32_split.cu),
    // laid out K-major; plain fp32 operands never reach kind::tf32 directly.
    if (!g.tf32_split || g.sa_k != 1 || g.sb_k != 1 || g.n_peers > 0) {
      if (why) *why = "fp32 reaches tcgen05 only as TF32-split, K-major operands (no all-gather)";
      return false;
    }
  } else if (g.dtype != KF_FP16 && g.dtype != KF_BF16) {
    if (why) *why = "unknown dtype for tcgen05";
    return false;
  }
  if (operand_major(g.a, g.sa_m, g.sa_k, g.M, g.K) < 0 ||
      operand_major(g.b, g.sb_n, g.sb_k, g.N, g.K) < 0) {
    if (why)
      *why =
          "operand strides/pointers are not TMA-describable (16-byte aligned base and row "
          "stride, K >= 8)";
    return false;
  }
  return true;
}

int query_tcgen05_config(int dtype, const kf_gemm_config& cfg, int64_t* smem_bytes,
                         int32_t* tmem_cols) {
  std::string why;
  if (dtype != KF_FP16 && dtype != KF_BF16 && dtype != KF_FP32)
    return set_error(KF_ERR_INVALID_CONFIG, "unknown dtype for tcgen05");
  int rc = validate_config(cfg, 0, dtype, &why);
  if (rc != KF_OK) return set_error(rc, why);
  const int64_t smem =
      smem_bytes_for(cfg.block_n, cfg.block_k, cfg.stages, cta_group_of(cfg), stage_elem_bytes(dtype));
  if (smem_bytes) *smem_bytes = smem;
  if (tmem_cols) *tmem_cols = static_cast<int32_t>(tmem_cols_for(cfg.block_n));
  if (smem > 232448)
    return set_error(KF_ERR_INVALID_CONFIG,
                     "shared memory " + std::to_string(smem) + " B exceeds 227 KiB per CTA");
  return KF_OK;
}

int64_t gemm_tcgen05_workspace_bytes(const GemmArgs& g, const kf_gemm_config& cfg,
                                     const DeviceInfo& dev) {
  (void)g;
  if (cfg.stream_k != 1) return 0;
  // counters, then two fp32 partial tiles (128 rows x BLOCK_N) per CTA
  const int grid = cfg.num_ctas > 0 ? cfg.num_ctas : dev.sm_count;
  return SK_COUNTER_BYTES + 2LL * grid * cfg.block_n * BM * 4;
}

namespace {

// Per (kernel, dynamic shared memory, device): how many SM-pair clusters fit
// at once (-1 until asked).
struct LaunchFacts {
  int pair_clusters = -1;
};

// The kernel's dynamic shared-memory limit only ever rises: a launch that asks
// for more than the largest request so far raises it, a smaller one leaves it
// (one kernel serves several stage counts and tile widths).
cudaError_t launch_facts(void* fn, int64_t smem, LaunchFacts** out) {
  static std::mutex mu;
  static std::map<std::tuple<void*, int64_t, int>, LaunchFacts> facts;
  static std::map<std::pair<void*, int>, int64_t> smem_limit;
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return err;
  std::lock_guard<std::mutex> lock(mu);
  int64_t& limit = smem_limit[std::make_pair(fn, device)];
  if (smem > limit) {
    err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (err != cudaSuccess) return err;
    limit = smem;
  }
  *out = &facts[std::make_tuple(fn, smem, device)];
  return cudaSuccess;
}

}  // namespace

int launch_gemm_tcgen05(const GemmArgs& g, const kf_gemm_config& cfg, const DeviceInfo& dev,
                        cudaStream_t stream) {
  std::string why;
  if (!tcgen05_operands_ok(g, &why)) return set_error(KF_ERR_UNALIGNED, why);
  const bool swap = cfg.swap_ab == 1;
  const View v = make_view(g, swap);
  const int a_major = operand_major(v.a, v.sa_r, v.sa_k, v.M, g.K);
  const int b_major = operand_major(v.b, v.sb_c, v.sb_k, v.N, g.K);
  if (a_major < 0 || b_major < 0) return set_error(KF_ERR_UNALIGNED, "operands not TMA-describable");
  int rc = validate_config(cfg, b_major, g.dtype, &why);
  if (rc != KF_OK) return set_error(rc, why);
  if (g.dtype == KF_FP32 && (a_major != 0 || b_major != 0))
    return set_error(KF_ERR_UNALIGNED, "TF32 operands must be K-major");
  if (v.M > INT32_MAX || v.N > INT32_MAX || g.K > INT32_MAX)
    return set_error(KF_ERR_UNSUPPORTED, "dimensions above 2^31 are not supported");

  const int cg = cta_group_of(cfg);
  const int bn = cfg.block_n, bk = cfg.block_k, S = cfg.stages;
  const int b_rows = bn / cg;
  const int elem = elem_bytes(g.dtype);
  const uint32_t atom = static_cast<uint32_t>(128 / elem);
  // The staged all-gather epilogue needs unit column stride and 16-byte
  // aligned rows in C and in every peer copy.
  bool peer_stage = g.n_peers > 0 && v.sc_c == 1 && (v.sc_r * 2) % 16 == 0 &&
                    (reinterpret_cast<uintptr_t>(g.c) & 15u) == 0;
  for (int i = 0; i < g.n_peers; ++i)
    peer_stage = peer_stage && (reinterpret_cast<uintptr_t>(g.peers[i]) & 15u) == 0;
  const int64_t smem = smem_bytes_for(bn, bk, S, cg, stage_elem_bytes(g.dtype), peer_stage);
  if (smem > dev.max_smem_optin)
    return set_error(KF_ERR_INVALID_CONFIG, "shared memory " + std::to_string(smem) +
                                                " B exceeds the device limit of " +
                                                std::to_string(dev.max_smem_optin));
  const int64_t smem_request = smem < MIN_SMEM_PER_CTA ? MIN_SMEM_PER_CTA : smem;

  CUtensorMap tm_a, tm_b, tm_b_half;
  // TF32 split operands: rows of two K-segments (small, big), both mapped
  const uint64_t k_extent = g.tf32_split ? 2 * static_cast<uint64_t>(g.K) : static_cast<uint64_t>(g.K);
  rc = a_major == 0 ? encode_map(&tm_a, g.dtype, v.a, k_extent, v.M, v.sa_r, atom, BM)
                    : encode_map(&tm_a, g.dtype, v.a, v.M, g.K, v.sa_k, atom, bk);
  if (rc != KF_OK) return rc;
  rc = b_major == 0 ? encode_map(&tm_b, g.dtype, v.b, k_extent, v.N, v.sb_c, atom, b_rows)
                    : encode_map(&tm_b, g.dtype, v.b, v.N, g.K, v.sb_k, atom, bk);
  if (rc != KF_OK) return rc;
  // Half-width tail tiles: an N/2 MMA needs N/2 a multiple of 16 per CTA pair
  // share, and MN-major B boxes stay 64 columns wide.
  const bool split_ok = cfg.stream_k == 3 && (bn / 2) % (16 * cg) == 0 &&
                        (b_major == 0 || (b_rows / 2) % 64 == 0);
  tm_b_half = tm_b;
  if (split_ok && b_major == 0) {
    rc = encode_map(&tm_b_half, g.dtype, v.b, k_extent, v.N, v.sb_c, atom, b_rows / 2);
    if (rc != KF_OK) return rc;
  }

  TcParams p{};
  p.M = static_cast<int>(v.M);
  p.N = static_cast<int>(v.N);
  p.K = static_cast<int>(g.K);
  p.bn = bn;
  p.bk = bk;
  p.stages = S;
  p.group_m = cfg.group_m;
  p.a_mn = a_major;
  p.b_mn = b_major;
  p.tiles_m = static_cast<int>(ceil_div(v.M, BM * cg));
  p.tiles_n = static_cast<int>(ceil_div(v.N, bn));
  p.kb_per_tile = static_cast<int>(ceil_div(g.K, bk));
  const long long tiles = static_cast<long long>(p.tiles_m) * p.tiles_n;
  p.total_iters = tiles * p.kb_per_tile;
  p.c = g.c;
  p.sc_r = v.sc_r;
  p.sc_c = v.sc_c;
  p.bias = g.bias;
  p.bias_on_rows = v.bias_on_rows ? 1 : 0;
  p.n_peers = g.n_peers;
  for (int i = 0; i < g.n_peers; ++i) p.peers[i] = g.peers[i];
  OutMaps<true> out_maps{};
  p.peer_stage = 0;
  if (peer_stage) {
    // TMA stores (library choice) unless the config asks for thread stores.
    p.peer_stage = cfg.epi_store == 1 ? 1 : 2;
    if (p.peer_stage == 2) {
      rc = encode_map(&out_maps.m[0], g.dtype, g.c, static_cast<uint64_t>(v.N), static_cast<uint64_t>(v.M),
                      v.sc_r, 64, 32);
      for (int i = 0; rc == KF_OK && i < g.n_peers; ++i)
        rc = encode_map(&out_maps.m[1 + i], g.dtype, g.peers[i], static_cast<uint64_t>(v.N),
                        static_cast<uint64_t>(v.M), v.sc_r, 64, 32);
      if (rc != KF_OK) return rc;
    }
  }
  p.status = dev.status;
  const uint32_t fmt = g.dtype == KF_FP32 ? 2u : g.dtype == KF_BF16 ? 1u : 0u;
  p.idesc = instr_desc_f16(fmt, static_cast<uint32_t>(a_major), static_cast<uint32_t>(b_major), BM * cg,
                           static_cast<uint32_t>(bn));
  p.idesc_half = instr_desc_f16(fmt, static_cast<uint32_t>(a_major), static_cast<uint32_t>(b_major),
                                BM * cg, static_cast<uint32_t>(bn / 2));
  p.promote_kb = g.dtype == KF_FP32 ? (TF32_PROMOTE_K + bk - 1) / bk : 0;
  p.tf32_kp = g.dtype == KF_FP32 ? static_cast<int>(g.K) : 0;
  const int parts = g.dtype == KF_FP32 ? 2 : 1;
  p.a_stage_bytes = static_cast<uint32_t>(BM * bk * elem * parts);
  p.b_stage_bytes = static_cast<uint32_t>(b_rows * bk * elem * parts);
  p.tmem_cols = tmem_cols_for(bn);

  void* fn = pick_kernel(g.dtype, g.epilogue, cg, g.n_peers > 0);
  // The attribute and the pair occupancy depend only on (kernel, shared memory,
  // device): looked up once and kept, since the driver calls cost more host
  // time per launch than a small GEMM takes on the GPU.
  LaunchFacts* facts = nullptr;
  cudaError_t err = launch_facts(fn, smem_request, &facts);
  if (err != cudaSuccess) return cuda_error(err, "cudaFuncSetAttribute(tcgen05 gemm)");

  cudaLaunchConfig_t lc{};
  lc.blockDim = dim3(NUM_THREADS);
  lc.dynamicSmemBytes = static_cast<size_t>(smem_request);
  lc.stream = stream;
  cudaLaunchAttribute attr[1];
  lc.attrs = attr;
  lc.numAttrs = 0;

  int units = cfg.num_ctas > 0 ? cfg.num_ctas / cg : dev.sm_count / cg;
  if (cg == 2) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    lc.numAttrs = 1;
    if (cfg.num_ctas <= 0) {
      // Persistent pairs: as many as can be resident at once (pairs must share a GPC).
      if (facts->pair_clusters < 0) {
        lc.gridDim = dim3(static_cast<unsigned>(2 * units));
        int clusters = 0;
        err = cudaOccupancyMaxActiveClusters(&clusters, fn, &lc);
        if (err != cudaSuccess) return cuda_error(err, "cudaOccupancyMaxActiveClusters");
        facts->pair_clusters = clusters;
      }
      const int clusters = facts->pair_clusters;
      if (clusters > 0 && clusters < units) units = clusters;
    }
  }
  // The schedule: whole tiles; all stream-K; or (split tail) whole tiles for
  // the full waves and the last partial wave as half-width tiles, which pays
  // when the halves still fit one round (2 x remainder <= units).
  long long dp = tiles;
  p.tail_halves = 0;
  if (cfg.stream_k == 1) {
    dp = 0;
  } else if (split_ok) {
    const long long rem = tiles % units;
    if (rem != 0 && 2 * rem <= units && tiles > units) {
      dp = tiles - rem;
      p.tail_halves = static_cast<int>(2 * rem);
    }
  }
  p.dp_tiles = dp;
  p.sk_base = dp * p.kb_per_tile;
  p.sk_iters = cfg.stream_k == 1 ? tiles * p.kb_per_tile : 0;
  p.stream_k = p.sk_iters > 0 ? 1 : 0;
  if (p.stream_k) {
    if (dp == 0 && units > p.sk_iters) units = static_cast<int>(p.sk_iters);
    const int64_t need = gemm_tcgen05_workspace_bytes(g, cfg, dev);
    if (g.workspace == nullptr || g.workspace_bytes < need)
      return set_error(KF_ERR_WORKSPACE, "stream-K needs " + std::to_string(need) +
                                             " bytes of zero-initialised workspace");
    if ((reinterpret_cast<uintptr_t>(g.workspace) & 255u) != 0)
      return set_error(KF_ERR_WORKSPACE, "workspace must be 256-byte aligned");
    if (tiles * cg > SK_MAX_TILES)
      return set_error(KF_ERR_INVALID_CONFIG, "stream-K takes at most " +
                                                  std::to_string(SK_MAX_TILES / cg) +
                                                  " output tiles; use whole tiles");
    // Counters first, at a fixed offset: every call finds them where the last
    // call left them (at zero), whatever its tile or grid size.
    p.counters = static_cast<int*>(g.workspace);
    p.partials = reinterpret_cast<float*>(static_cast<char*>(g.workspace) + SK_COUNTER_BYTES);
  } else {
    if (units > tiles) units = static_cast<int>(tiles);
  }
  if (units < 1) units = 1;
  lc.gridDim = dim3(static_cast<unsigned>(units * cg));

  void* args[] = {&tm_a, &tm_b, &tm_b_half, &p, &out_maps};
  err = cudaLaunchKernelExC(&lc, fn, args);
  if (err != cudaSuccess) return cuda_error(err, "launch(tcgen05 gemm)");
  return KF_OK;
}

}  // namespace kf
