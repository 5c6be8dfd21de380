// CUDA-core GEMM for everything the tcgen05 path cannot take: fp32 operands
// (tcgen05 has no IEEE-fp32 MMA, and TF32 misses the 1e-5 fp32 gate), and
// fp16/bf16 operands whose strides or base pointers no TMA tensor map can
// describe (odd K such as 4099 or 509, unaligned views).
//
// Classic two-level tiling: a CTA owns a BM x BN tile of C, stages BK-deep
// slices of A and B in shared memory as fp32 (double-buffered, next slice
// prefetched into registers while the current one is consumed), and each of
// its 256 threads accumulates a TM x TN sub-block with FFMA in fp32. Element
// loads are bounds-checked against M/N/K and honour arbitrary strides; the
// fused bias + GELU epilogue matches the tcgen05 kernel's.
//
// Reference: kernelforge/kernels/matmul.py:54-113 (same blocked algorithm,
// fp32 accumulation, masked tails) and fused_linear.py:94-104 (epilogue).
#include "kf_common.cuh"
#include "kf_internal.h"

namespace kf {
namespace {

struct SimtParams {
  const void* a;
  long long sa_m, sa_k;
  const void* b;
  long long sb_k, sb_n;
  void* c;
  long long sc_m, sc_n;
  int M, N, K;
  const void* bias;
  int a_m_fast, b_n_fast;  // which index varies fastest across threads when loading
};

template <typename T, int BM, int BN, int BK, int TM, int TN, int EPI>
__global__ void __launch_bounds__((BM / TM) * (BN / TN))
    simt_gemm_kernel(const SimtParams p) {
  constexpr int THREADS = (BM / TM) * (BN / TN);
  constexpr int A_PER_THREAD = BM * BK / THREADS;
  constexpr int B_PER_THREAD = BK * BN / THREADS;
  constexpr int TX = BN / TN;  // threads along N
  static_assert(A_PER_THREAD >= 1 && B_PER_THREAD >= 1, "tile too small for the CTA");

  __shared__ float As[2][BK][BM];
  __shared__ float Bs[2][BK][BN];

  const int tid = threadIdx.x;
  const int tx = tid % TX;
  const int ty = tid / TX;
  const int m0 = blockIdx.y * BM;
  const int n0 = blockIdx.x * BN;
  const T* A = static_cast<const T*>(p.a);
  const T* B = static_cast<const T*>(p.b);

  float a_reg[A_PER_THREAD];
  float b_reg[B_PER_THREAD];

  auto load_a = [&](int k0) {
#pragma unroll
    for (int r = 0; r < A_PER_THREAD; ++r) {
      const int e = tid + r * THREADS;
      const int mi = p.a_m_fast ? e % BM : e / BK;
      const int ki = p.a_m_fast ? e / BM : e % BK;
      const int m = m0 + mi, k = k0 + ki;
      a_reg[r] = (m < p.M && k < p.K) ? to_f32(A[m * p.sa_m + k * p.sa_k]) : 0.0f;
    }
  };
  auto load_b = [&](int k0) {
#pragma unroll
    for (int r = 0; r < B_PER_THREAD; ++r) {
      const int e = tid + r * THREADS;
      const int ni = p.b_n_fast ? e % BN : e / BK;
      const int ki = p.b_n_fast ? e / BN : e % BK;
      const int n = n0 + ni, k = k0 + ki;
      b_reg[r] = (n < p.N && k < p.K) ? to_f32(B[k * p.sb_k + n * p.sb_n]) : 0.0f;
    }
  };
  auto stash = [&](int buf) {
#pragma unroll
    for (int r = 0; r < A_PER_THREAD; ++r) {
      const int e = tid + r * THREADS;
      const int mi = p.a_m_fast ? e % BM : e / BK;
      const int ki = p.a_m_fast ? e / BM : e % BK;
      As[buf][ki][mi] = a_reg[r];
    }
#pragma unroll
    for (int r = 0; r < B_PER_THREAD; ++r) {
      const int e = tid + r * THREADS;
      const int ni = p.b_n_fast ? e % BN : e / BK;
      const int ki = p.b_n_fast ? e / BN : e % BK;
      Bs[buf][ki][ni] = b_reg[r];
    }
  };

  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.0f;

  load_a(0);
  load_b(0);
  stash(0);
  __syncthreads();

  const int k_tiles = (p.K + BK - 1) / BK;
  for (int kt = 0; kt < k_tiles; ++kt) {
    const int buf = kt & 1;
    const bool more = kt + 1 < k_tiles;
    if (more) {
      load_a((kt + 1) * BK);
      load_b((kt + 1) * BK);
    }
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float av[TM], bv[TN];
#pragma unroll
      for (int i = 0; i < TM; ++i) av[i] = As[buf][kk][ty + i * (BM / TM)];
#pragma unroll
      for (int j = 0; j < TN; ++j) bv[j] = Bs[buf][kk][tx + j * TX];
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (more) stash(buf ^ 1);
    __syncthreads();
  }

  T* C = static_cast<T*>(p.c);
  const T* bias = static_cast<const T*>(p.bias);
#pragma unroll
  for (int j = 0; j < TN; ++j) {
    const int n = n0 + tx + j * TX;
    if (n >= p.N) continue;
    const float bj = (EPI != KF_EPI_NONE) ? to_f32(bias[n]) : 0.0f;
#pragma unroll
    for (int i = 0; i < TM; ++i) {
      const int m = m0 + ty + i * (BM / TM);
      if (m < p.M) C[m * p.sc_m + n * p.sc_n] = from_f32<T>(apply_epilogue<EPI>(acc[i][j], bj));
    }
  }
}

template <typename T, int BM, int BN, int BK, int TM, int TN>
int launch_tile(const SimtParams& p, int epi, cudaStream_t stream) {
  constexpr int THREADS = (BM / TM) * (BN / TN);
  dim3 grid(static_cast<unsigned>((p.N + BN - 1) / BN), static_cast<unsigned>((p.M + BM - 1) / BM));
  dim3 block(THREADS);
  switch (epi) {
    case KF_EPI_NONE:
      simt_gemm_kernel<T, BM, BN, BK, TM, TN, KF_EPI_NONE><<<grid, block, 0, stream>>>(p);
      break;
    case KF_EPI_BIAS:
      simt_gemm_kernel<T, BM, BN, BK, TM, TN, KF_EPI_BIAS><<<grid, block, 0, stream>>>(p);
      break;
    case KF_EPI_BIAS_GELU_TANH:
      simt_gemm_kernel<T, BM, BN, BK, TM, TN, KF_EPI_BIAS_GELU_TANH><<<grid, block, 0, stream>>>(p);
      break;
    default:
      simt_gemm_kernel<T, BM, BN, BK, TM, TN, KF_EPI_BIAS_GELU_ERF><<<grid, block, 0, stream>>>(p);
      break;
  }
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return cuda_error(err, "launch(simt gemm)");
  return KF_OK;
}

template <typename T>
int launch_typed(const SimtParams& p, const kf_gemm_config& cfg, int epi, cudaStream_t stream) {
  if (cfg.block_m == 128 && cfg.block_n == 128 && cfg.block_k == 8)
    return launch_tile<T, 128, 128, 8, 8, 8>(p, epi, stream);
  if (cfg.block_m == 64 && cfg.block_n == 64 && cfg.block_k == 16)
    return launch_tile<T, 64, 64, 16, 4, 4>(p, epi, stream);
  if (cfg.block_m == 128 && cfg.block_n == 64 && cfg.block_k == 16)
    return launch_tile<T, 128, 64, 16, 8, 4>(p, epi, stream);
  return set_error(KF_ERR_INVALID_CONFIG,
                   "SIMT GEMM tiles are (BLOCK_M, BLOCK_N, BLOCK_K) in {(128,128,8), (64,64,16), "
                   "(128,64,16)}; got (" +
                       std::to_string(cfg.block_m) + "," + std::to_string(cfg.block_n) + "," +
                       std::to_string(cfg.block_k) + ")");
}

}  // namespace

int launch_gemm_simt(const GemmArgs& g, const kf_gemm_config& cfg, cudaStream_t stream) {
  if (g.M > INT32_MAX || g.N > INT32_MAX || g.K > INT32_MAX)
    return set_error(KF_ERR_UNSUPPORTED, "dimensions above 2^31 are not supported");
  SimtParams p{};
  p.a = g.a;
  p.sa_m = g.sa_m;
  p.sa_k = g.sa_k;
  p.b = g.b;
  p.sb_k = g.sb_k;
  p.sb_n = g.sb_n;
  p.c = g.c;
  p.sc_m = g.sc_m;
  p.sc_n = g.sc_n;
  p.M = static_cast<int>(g.M);
  p.N = static_cast<int>(g.N);
  p.K = static_cast<int>(g.K);
  p.bias = g.bias;
  p.a_m_fast = (g.sa_m == 1 && g.sa_k != 1) ? 1 : 0;
  p.b_n_fast = (g.sb_k == 1 && g.sb_n != 1) ? 0 : 1;
  switch (g.dtype) {
    case KF_FP16: return launch_typed<__half>(p, cfg, g.epilogue, stream);
    case KF_BF16: return launch_typed<__nv_bfloat16>(p, cfg, g.epilogue, stream);
    case KF_FP32: return launch_typed<float>(p, cfg, g.epilogue, stream);
    default: return set_error(KF_ERR_INVALID_ARGUMENT, "unknown dtype code");
  }
}

}  // namespace kf
