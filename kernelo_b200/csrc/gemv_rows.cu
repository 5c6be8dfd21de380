// Decode-shape GEMV on CUDA cores: y[m, n] = sum_k x[m, k] * w[n, k] for up to
// four rows of x and a weight whose rows are K-contiguous (nn.Linear's [N, K]).
//
// At M <= 4 the product is ~1 FLOP per weight byte, so the kernel's job is to
// stream W from HBM at full rate. Each warp takes R whole weight rows at a
// time (tiles of R rows, tile t then t + warps_in_grid, ...) and reads them as
// contiguous 512-byte warp loads, U per row in flight per lane, so every DRAM
// page is read front to back by one warp. x is staged once per CTA in shared
// memory as fp32; per 16-byte weight vector position a lane reads the
// matching x values of each row m once (16-byte shared loads), converts the R
// weight vectors and accumulates with packed fp32x2 FMAs (sm_100
// `fma.rn.f32x2`). The row sums are reduced over the warp with shuffles and
// rounded once into y. With more rows of x the shared-memory reads of x
// outgrow the weight stream; those shapes take the tcgen05 GEMV.
//
// Replaces the reference's matmul launch at decode shapes
// (kernelforge/kernels/matmul.py:132-155 with M in {1, 4, 16}); fp32
// accumulation and one output rounding as in the reference's matmul.
#include "kf_common.cuh"
#include "kf_internal.h"
#include "rows_math.cuh"

namespace kf {
namespace {

constexpr int GEMV_MAX_WARPS = 32;

struct GemvRowsParams {
  const void* x;
  long long sx_m, sx_k;
  const void* w;
  long long sw_n;
  void* y;
  long long sy_m, sy_n;
  int M, N, K;
};

__device__ __forceinline__ uint64_t pack2(float a, float b) {
  return static_cast<uint64_t>(__float_as_uint(a)) |
         (static_cast<uint64_t>(__float_as_uint(b)) << 32);
}
__device__ __forceinline__ float2 unpack2(uint64_t v) {
  return make_float2(__uint_as_float(static_cast<uint32_t>(v)),
                     __uint_as_float(static_cast<uint32_t>(v >> 32)));
}
// d = a * b + c on two fp32 lanes at once (round to nearest, as fmaf).
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// The 16-byte weight vector as packed fp32 pairs.
template <typename T>
__device__ __forceinline__ void weight_pairs(const uint4& v, uint64_t* out) {
  constexpr int VE = RowVec<T>::VE;
  float f[VE];
  to_floats<T>(v, f);
#pragma unroll
  for (int i = 0; i < VE / 2; ++i) out[i] = pack2(f[2 * i], f[2 * i + 1]);
}

// MP: rows of x the kernel is compiled for (M rounded up); R: weight rows a
// warp takes at once (each x value read from shared memory serves all R);
// U: 16-byte weight vectors per row a lane keeps in flight.
//
// Shared memory holds x as fp32 in PLANES planes per row m: plane p holds
// elements 4p..4p+3 of every 16-byte weight vector, so the lanes of a warp,
// which take consecutive vectors, read consecutive 16-byte words (no bank
// conflicts). The K % VE tail elements follow the planes.
template <typename T, int MP, int R, int U, int WARPS>
__global__ void __launch_bounds__(32 * WARPS, 1) gemv_rows_kernel(const GemvRowsParams p) {
  constexpr int VE = RowVec<T>::VE;
  constexpr int PAIRS = VE / 2;
  constexpr int PLANES = VE / 4;
  extern __shared__ float4 xs4[];
  const int K = p.K;
  const int nvec = K / VE;  // whole 16-byte vectors of a row
  const int tail = K - nvec * VE;
  float* planes = reinterpret_cast<float*>(xs4);                // [MP][PLANES][nvec][4]
  float* xtail = planes + static_cast<size_t>(MP) * nvec * VE;  // [MP][VE]
  {
    // Every CTA stages x before its first weight row, so the loads are issued
    // in batches of independent 16-byte (or, for strided x, 8 scalar) loads:
    // one memory latency per batch rather than one per element.
    const T* x = static_cast<const T*>(p.x);
    const bool xvec = p.sx_k == 1 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0 &&
                      ((p.sx_m * static_cast<long long>(sizeof(T))) & 15) == 0;
    const int total = MP * nvec;  // 16-byte vectors of x, rows >= M read as zero
    constexpr int BATCH = 4;
    for (int i0 = threadIdx.x; i0 < total; i0 += BATCH * blockDim.x) {
      uint4 q[BATCH];
#pragma unroll
      for (int b = 0; b < BATCH; ++b) {
        const int i = i0 + b * blockDim.x;
        const int m = i / nvec, v = i - m * nvec;
        q[b] = make_uint4(0u, 0u, 0u, 0u);
        if (i < total && m < p.M) {
          const T* src = x + m * p.sx_m;
          if (xvec) {
            q[b] = *reinterpret_cast<const uint4*>(src + v * VE);
          } else {
            T e[VE];
#pragma unroll
            for (int k = 0; k < VE; ++k) e[k] = src[(v * VE + k) * p.sx_k];
            memcpy(&q[b], e, 16);
          }
        }
      }
#pragma unroll
      for (int b = 0; b < BATCH; ++b) {
        const int i = i0 + b * blockDim.x;
        if (i < total) {
          const int m = i / nvec, v = i - m * nvec;
          float f[VE];
          to_floats<T>(q[b], f);
#pragma unroll
          for (int pl = 0; pl < PLANES; ++pl)
            *reinterpret_cast<float4*>(planes + ((m * PLANES + pl) * nvec + v) * 4) =
                make_float4(f[4 * pl], f[4 * pl + 1], f[4 * pl + 2], f[4 * pl + 3]);
        }
      }
    }
    for (int i = threadIdx.x; i < MP * VE; i += blockDim.x) {
      const int m = i / VE, t = i - m * VE;
      xtail[i] = (m < p.M && t < tail) ? to_f32(x[m * p.sx_m + (nvec * VE + t) * p.sx_k]) : 0.0f;
    }
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = (p.N + R - 1) / R;
  const int warps = gridDim.x * WARPS;
  for (int tile = blockIdx.x * WARPS + warp; tile < tiles; tile += warps) {
    const int n0 = tile * R;
    const T* wr[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int n = n0 + r < p.N ? n0 + r : p.N - 1;  // clamped: the row is read, not written
      wr[r] = static_cast<const T*>(p.w) + static_cast<long long>(n) * p.sw_n;
    }
    uint64_t acc[R][MP];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int m = 0; m < MP; ++m) acc[r][m] = 0;
    for (int v0 = lane; v0 < nvec; v0 += 32 * U) {
      uint4 raw[R][U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int v = v0 + 32 * u;
#pragma unroll
        for (int r = 0; r < R; ++r)
          if (v < nvec) raw[r][u] = __ldcs(reinterpret_cast<const uint4*>(wr[r]) + v);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int v = v0 + 32 * u;
        if (v < nvec) {
          uint64_t xp[MP][PAIRS];
#pragma unroll
          for (int m = 0; m < MP; ++m) {
#pragma unroll
            for (int pl = 0; pl < PLANES; ++pl) {
              const ulonglong2 q = *reinterpret_cast<const ulonglong2*>(
                  planes + ((m * PLANES + pl) * nvec + v) * 4);
              xp[m][2 * pl] = q.x;
              xp[m][2 * pl + 1] = q.y;
            }
          }
#pragma unroll
          for (int r = 0; r < R; ++r) {
            uint64_t wp[PAIRS];
            weight_pairs<T>(raw[r][u], wp);
#pragma unroll
            for (int m = 0; m < MP; ++m)
#pragma unroll
              for (int i = 0; i < PAIRS; ++i) acc[r][m] = ffma2(wp[i], xp[m][i], acc[r][m]);
          }
        }
      }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float sum[MP];
#pragma unroll
      for (int m = 0; m < MP; ++m) {
        const float2 a = unpack2(acc[r][m]);
        sum[m] = a.x + a.y;
      }
      if (lane < tail) {  // scalar tail: one element per lane
        const float wk = to_f32(wr[r][nvec * VE + lane]);
#pragma unroll
        for (int m = 0; m < MP; ++m) sum[m] = fmaf(wk, xtail[m * VE + lane], sum[m]);
      }
#pragma unroll
      for (int m = 0; m < MP; ++m) sum[m] = warp_sum(sum[m]);
      if (lane < p.M && n0 + r < p.N) {
        float s = sum[0];
#pragma unroll
        for (int m = 1; m < MP; ++m)
          if (lane == m) s = sum[m];
        static_cast<T*>(p.y)[lane * p.sy_m + static_cast<long long>(n0 + r) * p.sy_n] =
            from_f32<T>(s);
      }
    }
  }
}

int round_rows(int m) { return m <= 1 ? 1 : m <= 2 ? 2 : 4; }

size_t gemv_rows_smem(int mp, int64_t K, int elem) {
  const int ve = 16 / elem;
  return static_cast<size_t>(mp) * (K / ve * ve + ve) * sizeof(float);
}

template <typename T, int MP, int R, int U, int WARPS>
int launch_shape(const GemvRowsParams& p, const kf_gemm_config& cfg, const DeviceInfo& dev,
                 cudaStream_t stream) {
  auto fn = gemv_rows_kernel<T, MP, R, U, WARPS>;
  const size_t smem = gemv_rows_smem(MP, p.K, sizeof(T));
  cudaError_t err =
      cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (err != cudaSuccess) return cuda_error(err, "cudaFuncSetAttribute(gemv rows)");
  int occ = 0;
  err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, 32 * WARPS, smem);
  if (err != cudaSuccess) return cuda_error(err, "occupancy(gemv rows)");
  if (occ < 1) return set_error(KF_ERR_INVALID_CONFIG, "gemv rows kernel cannot launch");
  int64_t grid = cfg.num_ctas > 0 ? cfg.num_ctas : static_cast<int64_t>(dev.sm_count) * occ;
  const int64_t needed = ceil_div(ceil_div(p.N, R), WARPS);
  if (grid > needed) grid = needed;
  fn<<<static_cast<unsigned>(grid), 32 * WARPS, smem, stream>>>(p);
  err = cudaGetLastError();
  if (err != cudaSuccess) return cuda_error(err, "launch(gemv rows)");
  return KF_OK;
}

// Launch shapes (warps per CTA, R rows per warp, U vectors per row in flight)
// compiled for each row count; config block_m / block_n / block_k select one,
// zero picks the default (the first of each list).
template <typename T, int MP>
int launch_mp(const GemvRowsParams& p, const kf_gemm_config& cfg, const DeviceInfo& dev,
              cudaStream_t stream) {
  const int warps = cfg.block_m, r = cfg.block_n, u = cfg.block_k;
  auto is = [&](int w, int rr, int uu) {
    return (warps == 0 && r == 0 && u == 0) || (warps == w && r == rr && u == uu);
  };
  if constexpr (MP == 1) {
    if (is(16, 1, 16)) return launch_shape<T, MP, 1, 16, 16>(p, cfg, dev, stream);
    if (is(32, 1, 8)) return launch_shape<T, MP, 1, 8, 32>(p, cfg, dev, stream);
    if (is(32, 1, 4)) return launch_shape<T, MP, 1, 4, 32>(p, cfg, dev, stream);
    if (is(32, 2, 4)) return launch_shape<T, MP, 2, 4, 32>(p, cfg, dev, stream);
  } else {
    if (is(16, 2, 8)) return launch_shape<T, MP, 2, 8, 16>(p, cfg, dev, stream);
    if (is(32, 2, 4)) return launch_shape<T, MP, 2, 4, 32>(p, cfg, dev, stream);
    if (is(32, 2, 2)) return launch_shape<T, MP, 2, 2, 32>(p, cfg, dev, stream);
    if (is(32, 4, 2)) return launch_shape<T, MP, 4, 2, 32>(p, cfg, dev, stream);
    if (is(32, 1, 4)) return launch_shape<T, MP, 1, 4, 32>(p, cfg, dev, stream);
  }
  return set_error(KF_ERR_INVALID_CONFIG,
                   "warp-per-row GEMV: no compiled shape with " + std::to_string(warps) +
                       " warps, " + std::to_string(r) + " rows per warp, " + std::to_string(u) +
                       " vectors in flight for " + std::to_string(MP) + " rows of x");
}

template <typename T>
int launch_typed(const GemvRowsParams& p, const kf_gemm_config& cfg, const DeviceInfo& dev,
                 cudaStream_t stream) {
  switch (round_rows(p.M)) {
    case 1: return launch_mp<T, 1>(p, cfg, dev, stream);
    case 2: return launch_mp<T, 2>(p, cfg, dev, stream);
    default: return launch_mp<T, 4>(p, cfg, dev, stream);
  }
}

}  // namespace

bool gemv_rows_supported(int dtype, const void* w, int64_t sw_n, int64_t sw_k, int64_t M,
                         int64_t N, int64_t K, int max_smem_optin, std::string* why) {
  const int elem = dtype == KF_FP32 ? 4 : 2;
  if (M < 1 || M > GEMV_ROWS_MAX_M) {
    if (why) *why = "the warp-per-row GEMV takes 1.." + std::to_string(GEMV_ROWS_MAX_M) + " rows of x";
    return false;
  }
  if (N > INT32_MAX || K > INT32_MAX) {
    if (why) *why = "dimensions above 2^31";
    return false;
  }
  if (sw_k != 1 && K > 1) {
    if (why) *why = "weight rows must be K-contiguous ([N, K] with unit stride along K)";
    return false;
  }
  if ((reinterpret_cast<uintptr_t>(w) & 15u) != 0 || ((sw_n * elem) & 15) != 0) {
    if (why) *why = "weight rows must start on 16-byte boundaries";
    return false;
  }
  if (static_cast<int64_t>(gemv_rows_smem(round_rows(static_cast<int>(M)), K, elem)) > max_smem_optin) {
    if (why) *why = "x does not fit shared memory as fp32";
    return false;
  }
  return true;
}

int launch_gemv_rows(int dtype, const void* x, int64_t sx_m, int64_t sx_k, const void* w,
                     int64_t sw_n, void* y, int64_t sy_m, int64_t sy_n, int64_t M, int64_t N,
                     int64_t K, const kf_gemm_config& cfg, const DeviceInfo& dev,
                     cudaStream_t stream) {
  GemvRowsParams p{};
  p.x = x;
  p.sx_m = sx_m;
  p.sx_k = sx_k;
  p.w = w;
  p.sw_n = sw_n;
  p.y = y;
  p.sy_m = sy_m;
  p.sy_n = sy_n;
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  switch (dtype) {
    case KF_FP16: return launch_typed<__half>(p, cfg, dev, stream);
    case KF_BF16: return launch_typed<__nv_bfloat16>(p, cfg, dev, stream);
    case KF_FP32: return launch_typed<float>(p, cfg, dev, stream);
  }
  return set_error(KF_ERR_INVALID_ARGUMENT, "unknown dtype code");
}

}  // namespace kf
