// Decode-shape GEMM against a B whose rows are N-contiguous -- the reference's
// row-major (K, N) operand (kernelforge/kernels/matmul.py:132-155 at M in
// {1, 4, 16}): y[m, n] = epi(sum_k x[m, k] b[k, n]) for M <= 8, any dtype.
//
// At a handful of rows of x the product is ~M FLOP per byte of B, so the job
// is to stream B from HBM at full rate. The 16-row tile GEMV and the
// warp-per-row GEMV stream K-contiguous weight rows; here a row of B runs
// along N instead, so the kernel walks B row by row and gives each lane a
// fixed 16-byte vector of columns:
//
//   * a CTA of 8 warps owns a strip of 32 x VE columns (VE = 16 bytes of
//     elements); lane j always reads columns [strip + j*VE, +VE), so every
//     warp load is 512 contiguous bytes of one row of B;
//   * the grid splits K over S CTAs per strip (enough CTAs for every SM), and
//     a CTA deals its K rows to its warps round-robin, four rows in flight
//     per lane;
//   * x's rows for the CTA's K range are staged once in shared memory as
//     fp32, [k][m], and read back as broadcasts;
//   * each lane keeps MR x VE fp32 sums, accumulated with packed fp32x2 FMAs;
//     the 8 warps' sums meet in shared memory (a halving tree);
//   * with S > 1 every CTA writes its strip's partial sums to the workspace,
//     and the last of the strip's S CTAs to arrive (an arrival counter per
//     strip) adds all S partials in split order -- so results do not depend on
//     arrival order -- applies the epilogue (bias, GELU) and rounds once.
//     It resets the counter, leaving the workspace ready for the next call.
//
// Nothing waits on another CTA: the last arrival does the final sum.
#include "kf_common.cuh"
#include "kf_internal.h"
#include "rows_math.cuh"

namespace kf {
namespace {

constexpr int COLS_WARPS = 8;
constexpr int COLS_THREADS = COLS_WARPS * 32;
constexpr int COLS_UNROLL = 4;

struct GemvColsParams {
  const void* x;
  long long sx_m, sx_k;
  const void* b;
  long long sb_k;  // row stride of B (its columns are contiguous)
  void* y;
  long long sy_m, sy_n;
  const void* bias;
  int M, N, K;
  int splits;        // S: CTAs along K per strip
  float* partials;   // [S][M][N] fp32 (S > 1)
  int* counters;     // one per strip (S > 1)
};

template <typename T>
__device__ __forceinline__ void vec_to_f32(const uint4& v, float* f) {
  to_floats<T>(v, f);
}

template <typename T, int MR, int EPI>
__global__ void __launch_bounds__(COLS_THREADS) gemv_cols_kernel(const GemvColsParams p) {
  constexpr int VE = 16 / static_cast<int>(sizeof(T));
  constexpr int ACC = MR * VE;
  extern __shared__ __align__(16) float smem[];
  // [0, red): the reduction buffer of 4 warps; [red, ...): x as fp32 [k][MR]
  float* red = smem;
  float* xs = smem + 4 * ACC * 32;
  __shared__ unsigned last_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int strip = blockIdx.x, split = blockIdx.y;
  const int col = (strip * 32 + lane) * VE;
  const bool col_ok = col < p.N;
  const int k0 = static_cast<int>(static_cast<long long>(p.K) * split / p.splits);
  const int k1 = static_cast<int>(static_cast<long long>(p.K) * (split + 1) / p.splits);

  // x[:, k0:k1] -> shared memory as fp32, [k][m] (rows beyond M are zero)
  const T* x = static_cast<const T*>(p.x);
  for (int i = threadIdx.x; i < (k1 - k0) * MR; i += COLS_THREADS) {
    const int k = k0 + i / MR, m = i % MR;
    xs[i] = m < p.M ? to_f32(x[m * p.sx_m + static_cast<long long>(k) * p.sx_k]) : 0.0f;
  }
  __syncthreads();

  float acc[ACC];
#pragma unroll
  for (int i = 0; i < ACC; ++i) acc[i] = 0.0f;
  const T* bcol = static_cast<const T*>(p.b) + col;
  for (int kb = k0 + warp; kb < k1; kb += COLS_WARPS * COLS_UNROLL) {
    uint4 v[COLS_UNROLL];
#pragma unroll
    for (int u = 0; u < COLS_UNROLL; ++u) {
      const int k = kb + u * COLS_WARPS;
      v[u] = (col_ok && k < k1)
                 ? __ldcs(reinterpret_cast<const uint4*>(bcol + static_cast<long long>(k) * p.sb_k))
                 : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < COLS_UNROLL; ++u) {
      const int k = kb + u * COLS_WARPS;
      if (k >= k1) break;
      float f[VE];
      vec_to_f32<T>(v[u], f);
      const float* xk = xs + (k - k0) * MR;
#pragma unroll
      for (int m = 0; m < MR; ++m) {
        const float xm = xk[m];
        const uint64_t x2 = f2_splat(xm);
#pragma unroll
        for (int e = 0; e < VE; e += 2) {
          const uint64_t s = f2_fma(f2_pack(f[e], f[e + 1]), x2, f2_pack(acc[m * VE + e], acc[m * VE + e + 1]));
          const float2 r = f2_unpack(s);
          acc[m * VE + e] = r.x;
          acc[m * VE + e + 1] = r.y;
        }
      }
    }
  }

  // the 8 warps' sums: 4 -> 2 -> 1 rounds through a 4-warp buffer
#pragma unroll
  for (int half = COLS_WARPS / 2; half >= 1; half /= 2) {
    if (warp >= half && warp < 2 * half) {
#pragma unroll
      for (int i = 0; i < ACC; ++i) red[((warp - half) * ACC + i) * 32 + lane] = acc[i];
    }
    __syncthreads();
    if (warp < half) {
#pragma unroll
      for (int i = 0; i < ACC; ++i) acc[i] += red[(warp * ACC + i) * 32 + lane];
    }
    __syncthreads();
  }
  if (warp != 0) return;

  if (p.splits > 1) {
    // this split's partial sums, then the strip's arrival count
    if (col_ok) {
#pragma unroll
      for (int m = 0; m < MR; ++m) {
        if (m >= p.M) break;
        float4* dst = reinterpret_cast<float4*>(p.partials + (static_cast<size_t>(split) * p.M + m) * p.N + col);
#pragma unroll
        for (int e = 0; e < VE; e += 4)
          __stcg(dst + e / 4, make_float4(acc[m * VE + e], acc[m * VE + e + 1], acc[m * VE + e + 2],
                                          acc[m * VE + e + 3]));
      }
    }
    __threadfence();
    __syncwarp();
    if (lane == 0) last_flag = atomicAdd(p.counters + strip, 1) == p.splits - 1 ? 1u : 0u;
    __syncwarp();
    if (!last_flag) return;
    __threadfence();
    // the last arrival: all S partials in split order
#pragma unroll
    for (int i = 0; i < ACC; ++i) acc[i] = 0.0f;
    if (col_ok) {
      for (int s = 0; s < p.splits; ++s) {
#pragma unroll
        for (int m = 0; m < MR; ++m) {
          if (m >= p.M) break;
          const float4* src =
              reinterpret_cast<const float4*>(p.partials + (static_cast<size_t>(s) * p.M + m) * p.N + col);
#pragma unroll
          for (int e = 0; e < VE; e += 4) {
            const float4 q = __ldcg(src + e / 4);
            acc[m * VE + e] += q.x;
            acc[m * VE + e + 1] += q.y;
            acc[m * VE + e + 2] += q.z;
            acc[m * VE + e + 3] += q.w;
          }
        }
      }
    }
    if (lane == 0) p.counters[strip] = 0;
  }
  if (!col_ok) return;

  // epilogue and one rounding into y
  float bias[VE];
#pragma unroll
  for (int e = 0; e < VE; ++e) bias[e] = EPI != KF_EPI_NONE ? to_f32(static_cast<const T*>(p.bias)[col + e]) : 0.0f;
  T* y = static_cast<T*>(p.y);
#pragma unroll
  for (int m = 0; m < MR; ++m) {
    if (m >= p.M) break;
    float o[VE];
#pragma unroll
    for (int e = 0; e < VE; ++e) o[e] = apply_epilogue<EPI>(acc[m * VE + e], bias[e]);
    T* dst = y + m * p.sy_m + static_cast<long long>(col) * p.sy_n;
    if (p.sy_n == 1 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
      *reinterpret_cast<uint4*>(dst) = from_floats<T>(o);
    } else {
#pragma unroll
      for (int e = 0; e < VE; ++e) dst[static_cast<long long>(e) * p.sy_n] = from_f32<T>(o[e]);
    }
  }
}

template <typename T, int MR>
void* pick_cols_epi(int epi) {
  switch (epi) {
    case KF_EPI_NONE: return reinterpret_cast<void*>(&gemv_cols_kernel<T, MR, KF_EPI_NONE>);
    case KF_EPI_BIAS: return reinterpret_cast<void*>(&gemv_cols_kernel<T, MR, KF_EPI_BIAS>);
    case KF_EPI_BIAS_GELU_TANH: return reinterpret_cast<void*>(&gemv_cols_kernel<T, MR, KF_EPI_BIAS_GELU_TANH>);
    default: return reinterpret_cast<void*>(&gemv_cols_kernel<T, MR, KF_EPI_BIAS_GELU_ERF>);
  }
}

template <typename T>
void* pick_cols(int mr, int epi) {
  if (mr <= 1) return pick_cols_epi<T, 1>(epi);
  if (mr <= 2) return pick_cols_epi<T, 2>(epi);
  if (mr <= 4) return pick_cols_epi<T, 4>(epi);
  return pick_cols_epi<T, 8>(epi);
}

int elem_bytes(int dtype) { return dtype == KF_FP32 ? 4 : 2; }

}  // namespace

bool gemv_cols_supported(int dtype, const void* x, const void* b, int64_t sb_k, int64_t sb_n, int64_t M,
                         int64_t N, int64_t K, std::string* why) {
  const int eb = elem_bytes(dtype);
  const int ve = 16 / eb;
  auto no = [&](const char* reason) {
    if (why) *why = reason;
    return false;
  };
  if (M < 1 || M > GEMV_COLS_MAX_M) return no("the column GEMV takes 1..8 rows of x");
  if (sb_n != 1 || K < 1) return no("the column GEMV needs B's rows N-contiguous");
  if (N % ve != 0) return no("the column GEMV needs N a multiple of one 16-byte vector");
  if ((sb_k * eb) % 16 != 0 || (reinterpret_cast<uintptr_t>(b) & 15u) != 0)
    return no("the column GEMV needs a 16-byte-aligned B with 16-byte row pitch");
  (void)x;
  return true;
}

int gemv_cols_splits(int dtype, int64_t M, int64_t N, int64_t K, int sm_count) {
  const int ve = 16 / elem_bytes(dtype);
  const int64_t strips = (N + 32 * ve - 1) / (32 * ve);
  int64_t s = (4LL * sm_count + strips - 1) / strips;  // about four CTAs per SM
  const int64_t max_s = K / 64 > 0 ? K / 64 : 1;        // at least 64 rows of B per CTA
  if (s > max_s) s = max_s;
  if (s > 256) s = 256;
  if (s < 1) s = 1;
  (void)M;
  return static_cast<int>(s);
}

int64_t gemv_cols_workspace_bytes(int dtype, int64_t M, int64_t N, int64_t K, int sm_count) {
  const int s = gemv_cols_splits(dtype, M, N, K, sm_count);
  if (s <= 1) return 0;
  return SK_COUNTER_BYTES + static_cast<int64_t>(s) * M * N * 4;
}

int launch_gemv_cols(int dtype, const void* x, int64_t sx_m, int64_t sx_k, const void* b, int64_t sb_k,
                     void* y, int64_t sy_m, int64_t sy_n, int64_t M, int64_t N, int64_t K, int epilogue,
                     const void* bias, void* workspace, int64_t workspace_bytes, int sm_count,
                     cudaStream_t stream) {
  std::string why;
  if (!gemv_cols_supported(dtype, x, b, sb_k, 1, M, N, K, &why)) return set_error(KF_ERR_UNALIGNED, why);
  const int ve = 16 / elem_bytes(dtype);
  const int64_t strips = (N + 32 * ve - 1) / (32 * ve);
  if (strips > SK_COUNTER_BYTES / 4) return set_error(KF_ERR_UNSUPPORTED, "too many column strips");
  GemvColsParams p{};
  p.x = x;
  p.sx_m = sx_m;
  p.sx_k = sx_k;
  p.b = b;
  p.sb_k = sb_k;
  p.y = y;
  p.sy_m = sy_m;
  p.sy_n = sy_n;
  p.bias = bias;
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  int s = gemv_cols_splits(dtype, M, N, K, sm_count);
  if (s > 1 && (workspace == nullptr || workspace_bytes < SK_COUNTER_BYTES + static_cast<int64_t>(s) * M * N * 4))
    s = 1;  // no (or too little) workspace: one CTA per strip, no partials
  p.splits = s;
  if (s > 1) {
    if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
      return set_error(KF_ERR_WORKSPACE, "workspace must be 256-byte aligned");
    p.counters = static_cast<int*>(workspace);
    p.partials = reinterpret_cast<float*>(static_cast<char*>(workspace) + SK_COUNTER_BYTES);
  }
  const int mr = M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8;
  const int acc = mr * ve;
  const int64_t rows = (K + s - 1) / s + 1;
  const size_t smem = (static_cast<size_t>(4 * acc * 32) + static_cast<size_t>(rows) * mr) * sizeof(float);
  if (smem > 200 * 1024) return set_error(KF_ERR_UNSUPPORTED, "the column GEMV's K range per CTA is too long");
  void* fn = dtype == KF_FP16 ? pick_cols<__half>(mr, epilogue)
             : dtype == KF_BF16 ? pick_cols<__nv_bfloat16>(mr, epilogue)
                                : pick_cols<float>(mr, epilogue);
  cudaError_t err = cudaSuccess;
  if (smem > 48 * 1024) {
    err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (err != cudaSuccess) return cuda_error(err, "cudaFuncSetAttribute(gemv_cols)");
  }
  void* args[] = {&p};
  err = cudaLaunchKernel(fn, dim3(static_cast<unsigned>(strips), static_cast<unsigned>(s)), dim3(COLS_THREADS), args,
                         smem, stream);
  if (err != cudaSuccess) return cuda_error(err, "launch(gemv_cols_kernel)");
  return KF_OK;
}

}  // namespace kf
