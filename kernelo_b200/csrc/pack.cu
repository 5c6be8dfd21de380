// Operand packing for the tcgen05 GEMM: fp16/bf16 matrices whose layout a TMA
// tensor map cannot describe, copied into a pitched, 16-byte-aligned buffer.
//
// TMA needs a 16-byte-aligned base and row pitch. A row-major operand with
// K = 4099 (row pitch 8198 bytes), a B with N = 2053, or a view that starts at
// an odd column breaks that, and without packing such a problem can only run
// on CUDA cores -- at the prime sizes of the tuner sweep, several times slower
// than the tensor cores. Packing copies the operand once into the caller's
// workspace with the pitch rounded up to whole 16-byte vectors and the pad
// zero-filled (zeros along K add nothing to the products), then the tcgen05
// kernel runs on the copy. The copy keeps the operand's unit-stride dimension
// innermost, so a K-major operand stays K-major and an MN-major one MN-major.
//
// The copy reads every element once and writes it once: (outer x len) x 2
// bytes in, (outer x pitch) x 2 out. Worth it where the GEMM is compute-bound
// (gemm_common packs only when both M and N exceed 64); skinny problems keep
// the CUDA-core path, which streams the operand without a copy.
#include "kf_common.cuh"
#include "kf_internal.h"

namespace kf {
namespace {

// dst[r][c] = c < len ? src[r * s_outer + c * s_inner] : 0 for c < pitch
// (pitch a multiple of 8): each thread writes one 16-byte vector of 8
// elements. Threads of a warp cover consecutive vectors of one row, so both
// the 2-byte loads (the source row may start at any 2-byte address) and the
// 16-byte stores are coalesced.
__global__ void __launch_bounds__(256) pack16_kernel(const uint16_t* __restrict__ src, long long s_outer,
                                                     long long s_inner, long long outer, int len,
                                                     uint16_t* __restrict__ dst, int pitch) {
  const int vecs = pitch / 8;
  const int v = blockIdx.x * blockDim.x + threadIdx.x;
  if (v >= vecs) return;
  const int c0 = v * 8;
  for (long long r = blockIdx.y; r < outer; r += gridDim.y) {
    const uint16_t* row = src + r * s_outer;
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = c0 + 2 * j;
      const uint32_t lo = c < len ? __ldg(row + static_cast<long long>(c) * s_inner) : 0u;
      const uint32_t hi = c + 1 < len ? __ldg(row + static_cast<long long>(c + 1) * s_inner) : 0u;
      w[j] = lo | (hi << 16);
    }
    *reinterpret_cast<uint4*>(dst + r * pitch + c0) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// The inverse copy: dst[r * s_outer + c * s_inner] = src[r][c] for c < len;
// each thread reads one 16-byte vector of the pitched source and writes its
// elements with 2-byte stores (consecutive threads, consecutive columns).
__global__ void __launch_bounds__(256) unpack16_kernel(const uint16_t* __restrict__ src, int pitch, long long outer,
                                                       int len, uint16_t* __restrict__ dst, long long s_outer,
                                                       long long s_inner) {
  const int v = blockIdx.x * blockDim.x + threadIdx.x;
  const int c0 = v * 8;
  if (c0 >= len) return;
  for (long long r = blockIdx.y; r < outer; r += gridDim.y) {
    const uint4 q = *reinterpret_cast<const uint4*>(src + r * pitch + c0);
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
    uint16_t* row = dst + r * s_outer;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = c0 + j;
      if (c < len) row[static_cast<long long>(c) * s_inner] = static_cast<uint16_t>(w[j / 2] >> (16 * (j & 1)));
    }
  }
}

}  // namespace

PackedOperand plan_pack(const void* ptr, int64_t s_mn, int64_t s_k, int64_t mn, int64_t k, int64_t k_padded) {
  PackedOperand p;
  p.k_inner = !(s_mn == 1 && s_k != 1);  // the unit-stride dimension stays innermost
  p.len = p.k_inner ? k : mn;
  p.outer = p.k_inner ? mn : k_padded;
  p.pitch = ((p.k_inner ? k_padded : mn) + 7) / 8 * 8;
  if (p.pitch < 8) p.pitch = 8;
  p.bytes = (p.outer * p.pitch * 2 + 255) / 256 * 256;
  p.src = ptr;
  p.s_outer = p.k_inner ? s_mn : s_k;
  p.s_inner = p.k_inner ? s_k : s_mn;
  p.src_outer = p.k_inner ? mn : k;  // rows that exist in the source (the rest are zero)
  return p;
}

int launch_pack(const PackedOperand& p, void* dst, cudaStream_t stream) {
  if ((reinterpret_cast<uintptr_t>(dst) & 15u) != 0)
    return set_error(KF_ERR_WORKSPACE, "packing needs a 16-byte-aligned workspace");
  // rows past the source's extent (K padded to 8 for an MN-major copy) are zero
  if (p.outer > p.src_outer) {
    const cudaError_t err =
        cudaMemsetAsync(static_cast<uint16_t*>(dst) + p.src_outer * p.pitch, 0,
                        static_cast<size_t>((p.outer - p.src_outer) * p.pitch * 2), stream);
    if (err != cudaSuccess) return cuda_error(err, "cudaMemsetAsync(pack padding)");
  }
  if (p.src_outer == 0) return KF_OK;
  const int vecs = static_cast<int>(p.pitch / 8);
  dim3 grid(static_cast<unsigned>((vecs + 255) / 256),
            static_cast<unsigned>(p.src_outer < 65535 ? p.src_outer : 65535));
  pack16_kernel<<<grid, 256, 0, stream>>>(static_cast<const uint16_t*>(p.src), p.s_outer, p.s_inner,
                                          p.src_outer, static_cast<int>(p.len), static_cast<uint16_t*>(dst),
                                          static_cast<int>(p.pitch));
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return cuda_error(err, "launch(pack16_kernel)");
  return KF_OK;
}

PackedOperand plan_output_stage(void* c, int64_t sc_m, int64_t sc_n, int64_t m, int64_t n) {
  PackedOperand p;
  p.k_inner = true;
  p.outer = p.src_outer = m;
  p.len = n;
  p.pitch = (n + 7) / 8 * 8;
  p.bytes = (m * p.pitch * 2 + 255) / 256 * 256;
  p.src = c;
  p.s_outer = sc_m;
  p.s_inner = sc_n;
  return p;
}

int launch_unpack(const PackedOperand& p, const void* staged, cudaStream_t stream) {
  if (p.outer == 0 || p.len == 0) return KF_OK;
  const int vecs = static_cast<int>(p.pitch / 8);
  dim3 grid(static_cast<unsigned>((vecs + 255) / 256), static_cast<unsigned>(p.outer < 65535 ? p.outer : 65535));
  unpack16_kernel<<<grid, 256, 0, stream>>>(static_cast<const uint16_t*>(staged), static_cast<int>(p.pitch),
                                            p.outer, static_cast<int>(p.len),
                                            static_cast<uint16_t*>(const_cast<void*>(p.src)), p.s_outer,
                                            p.s_inner);
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return cuda_error(err, "launch(unpack16_kernel)");
  return KF_OK;
}

}  // namespace kf
