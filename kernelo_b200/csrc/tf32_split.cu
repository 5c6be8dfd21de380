// fp32 GEMM operands split for the 3xTF32 scheme on kind::tf32 tensor cores.
//
// An fp32 value x is written as big + small with big = tf32(x) (x rounded to
// TF32's 10 explicit mantissa bits) and small = tf32(x - big); x - big is
// exact in fp32, and small keeps the next 11 bits, so big + small carries 22
// of x's 24 significant bits. Then
//
//   a . b ~= a_small b_big + a_big b_small + a_big b_big
//
// (the dropped a_small b_small is below 2^-22 |a b|). TF32 x TF32 products
// are exact in fp32 and the tensor core accumulates in fp32, so the sum keeps
// fp32-level accuracy -- the reference's fp32 matmul is IEEE
// (kernelforge/kernels/matmul.py:93-106, input_precision="ieee") and its gate
// threshold for fp32 is 1e-5 (kernelforge/testing.py:31-35), which plain
// TF32 misses by about 100x.
//
// Each operand is copied once into the workspace as rows of two K-segments,
//
//   A' [M, 2 Kp] = [ A_small | A_big ]      B' [N, 2 Kp] = [ B_small | B_big ]
//
// K-major whatever the source layout (a row-major (K, N) B is transposed on
// the way through shared memory), which is the layout kind::tf32 reads; Kp is
// K rounded up to a 128-byte TMA atom (32 elements) with zeros. The tcgen05
// kernel loads both segments of a k-block into one ring stage and issues the
// three products' MMAs on them (small x big, big x small, big x big), so each
// byte crosses L2 and shared memory once per k-block. Rounding is
// cvt.rna.tf32.f32 (to nearest, ties away from zero).
#include "kf_common.cuh"
#include "kf_internal.h"

namespace kf {
namespace {

constexpr int SPLIT_TILE = 32;

__device__ __forceinline__ float to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// One 32 x 32 tile of the source (rows r0.., K positions k0..) per CTA of
// 32 x 8 threads: read along whichever index has unit stride, written along K.
__global__ void __launch_bounds__(256) tf32_split_kernel(const float* __restrict__ src, long long s_r,
                                                         long long s_k, long long rows, long long K,
                                                         float* __restrict__ dst, long long pitch,
                                                         long long kp) {
  __shared__ float tile[SPLIT_TILE][SPLIT_TILE + 1];
  const int tx = threadIdx.x, ty = threadIdx.y;
  const long long k0 = static_cast<long long>(blockIdx.x) * SPLIT_TILE;
  const long long r0 = static_cast<long long>(blockIdx.y) * SPLIT_TILE;
  const bool along_rows = s_k != 1 && s_r == 1;  // the rows' index is the contiguous one
#pragma unroll
  for (int i = 0; i < SPLIT_TILE / 8; ++i) {
    const int a = ty + 8 * i;
    if (along_rows) {
      const long long r = r0 + tx, k = k0 + a;
      tile[tx][a] = (r < rows && k < K) ? __ldg(src + k * s_k + r) : 0.0f;
    } else {
      const long long r = r0 + a, k = k0 + tx;
      tile[a][tx] = (r < rows && k < K) ? __ldg(src + r * s_r + k * s_k) : 0.0f;
    }
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < SPLIT_TILE / 8; ++i) {
    const int a = ty + 8 * i;
    const long long r = r0 + a;
    if (r >= rows) continue;
    const float x = tile[a][tx];
    const float big = to_tf32(x);
    const float small = to_tf32(x - big);
    float* row = dst + r * pitch + k0 + tx;
    row[0] = small;
    row[kp] = big;
  }
}

}  // namespace

SplitOperand plan_tf32_split(const void* src, int64_t s_r, int64_t s_k, int64_t rows, int64_t K) {
  SplitOperand s;
  s.src = src;
  s.s_r = s_r;
  s.s_k = s_k;
  s.rows = rows;
  s.K = K;
  s.kp = (K + SPLIT_TILE - 1) / SPLIT_TILE * SPLIT_TILE;
  s.pitch = 2 * s.kp;
  s.bytes = (rows * s.pitch * 4 + 255) / 256 * 256;
  return s;
}

int launch_tf32_split(const SplitOperand& s, void* dst, cudaStream_t stream) {
  if ((reinterpret_cast<uintptr_t>(dst) & 15u) != 0)
    return set_error(KF_ERR_WORKSPACE, "TF32 split buffer must be 16-byte aligned");
  if (s.rows == 0 || s.kp == 0) return KF_OK;
  const long long ktiles = s.kp / SPLIT_TILE;
  const long long rtiles = (s.rows + SPLIT_TILE - 1) / SPLIT_TILE;
  if (rtiles > 65535) return set_error(KF_ERR_UNSUPPORTED, "TF32 split: more than 2^21 rows");
  tf32_split_kernel<<<dim3(static_cast<unsigned>(ktiles), static_cast<unsigned>(rtiles)), dim3(32, 8), 0,
                      stream>>>(static_cast<const float*>(s.src), s.s_r, s.s_k, s.rows, s.K,
                                static_cast<float*>(dst), s.pitch, s.kp);
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return cuda_error(err, "launch(tf32 split)");
  return KF_OK;
}

}  // namespace kf
