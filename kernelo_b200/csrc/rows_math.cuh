// Arithmetic shared by the row kernels (rows.cu, rows_stream.cu).
//
// Both kernels are issue-bound unless the per-element work is a handful of
// instructions, so the helpers here work on whole 16-byte vectors:
//   * maxima are taken on packed pairs (half2 / bfloat162 max is exact, and
//     converting the final maximum to fp32 gives the fp32 maximum);
//   * conversions go pairwise (half2 -> float2);
//   * exponentials are one `ex2.approx.ftz.f32` each (PTX ISA: maximum relative
//     error 2^-22 over the full range; results below 2^-126 flush to zero,
//     which in a softmax sum whose largest term is 1 changes nothing).
// Statistics are fp32 and the output is rounded once, as in
// kernelforge/kernels/softmax.py:31-58 and kernelforge/kernels/rmsnorm.py:41-72.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <type_traits>

#include "kf_common.cuh"  // ex2_ftz, f2_*

namespace kf {

constexpr float kRowLog2e = 1.4426950408889634f;


template <typename P>
__device__ __forceinline__ P bitcast_pair(uint32_t u) {
  P p;
  memcpy(&p, &u, 4);
  return p;
}
template <typename P>
__device__ __forceinline__ uint32_t pair_bits(P p) {
  uint32_t u;
  memcpy(&u, &p, 4);
  return u;
}

// Operations on one 16-byte vector of T.
template <typename T>
struct RowVec;

template <>
struct RowVec<__half> {
  static constexpr int VE = 8;
  __device__ static uint4 lowest() {  // four packed -inf pairs
    return make_uint4(0xFC00FC00u, 0xFC00FC00u, 0xFC00FC00u, 0xFC00FC00u);
  }
  __device__ static uint32_t max2(uint32_t a, uint32_t b) {
    return pair_bits(__hmax2(bitcast_pair<__half2>(a), bitcast_pair<__half2>(b)));
  }
  __device__ static float2 to_f2(uint32_t u) { return __half22float2(bitcast_pair<__half2>(u)); }
  __device__ static uint32_t from_f2(float a, float b) { return pair_bits(__floats2half2_rn(a, b)); }
};

template <>
struct RowVec<__nv_bfloat16> {
  static constexpr int VE = 8;
  __device__ static uint4 lowest() {
    return make_uint4(0xFF80FF80u, 0xFF80FF80u, 0xFF80FF80u, 0xFF80FF80u);
  }
  __device__ static uint32_t max2(uint32_t a, uint32_t b) {
    return pair_bits(
        __hmax2(bitcast_pair<__nv_bfloat162>(a), bitcast_pair<__nv_bfloat162>(b)));
  }
  __device__ static float2 to_f2(uint32_t u) {
    return __bfloat1622float2(bitcast_pair<__nv_bfloat162>(u));
  }
  __device__ static uint32_t from_f2(float a, float b) {
    return pair_bits(__floats2bfloat162_rn(a, b));
  }
};

template <>
struct RowVec<float> {
  static constexpr int VE = 4;
  __device__ static uint4 lowest() {
    return make_uint4(0xFF800000u, 0xFF800000u, 0xFF800000u, 0xFF800000u);
  }
  __device__ static uint32_t max2(uint32_t a, uint32_t b) {
    return __float_as_uint(fmaxf(__uint_as_float(a), __uint_as_float(b)));
  }
  __device__ static float to_f1(uint32_t u) { return __uint_as_float(u); }
};

// Element-wise maximum of two vectors.
template <typename T>
__device__ __forceinline__ uint4 vmax(uint4 a, uint4 b) {
  using R = RowVec<T>;
  return make_uint4(R::max2(a.x, b.x), R::max2(a.y, b.y), R::max2(a.z, b.z), R::max2(a.w, b.w));
}

// Largest element of a vector, as fp32.
template <typename T>
__device__ __forceinline__ float hmax(uint4 v) {
  using R = RowVec<T>;
  const uint32_t m = R::max2(R::max2(v.x, v.y), R::max2(v.z, v.w));
  if constexpr (sizeof(T) == 4) {
    return __uint_as_float(m);
  } else {
    const float2 f = R::to_f2(m);
    return fmaxf(f.x, f.y);
  }
}

// The VE elements of a vector as fp32.
template <typename T>
__device__ __forceinline__ void to_floats(uint4 v, float* f) {
  if constexpr (sizeof(T) == 4) {
    f[0] = __uint_as_float(v.x);
    f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z);
    f[3] = __uint_as_float(v.w);
  } else {
    using R = RowVec<T>;
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 p = R::to_f2(w[i]);
      f[2 * i] = p.x;
      f[2 * i + 1] = p.y;
    }
  }
}

// VE fp32 values rounded once into a vector of T.
template <typename T>
__device__ __forceinline__ uint4 from_floats(const float* f) {
  if constexpr (sizeof(T) == 4) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                      __float_as_uint(f[3]));
  } else {
    using R = RowVec<T>;
    return make_uint4(R::from_f2(f[0], f[1]), R::from_f2(f[2], f[3]), R::from_f2(f[4], f[5]),
                      R::from_f2(f[6], f[7]));
  }
}

// ---- RMSNorm on 16-byte vectors with sm_100's mixed-precision FMA.
// `fma.rn.f32.{f16,bf16} d, a, b, c` multiplies two 16-bit values and adds an
// fp32 value with one rounding to fp32. A product of two 16-bit values is
// exact in fp32 (at most 22 significant bits), so x*x and x*gamma come out
// exact without converting either operand first: the sum of squares keeps the
// fp32 rounding of the reference's fp32 path (rmsnorm.py:130-143), and the
// output x * gamma * scale is rounded in fp32 once before the final rounding
// to T (the reference rounds (x*scale)*gamma twice in fp32).
template <typename T>
__device__ __forceinline__ float fma_mixed(uint16_t a, uint16_t b, float c) {
  float d;
  if constexpr (std::is_same_v<T, __half>) {
    asm("fma.rn.f32.f16 %0, %1, %2, %3;" : "=f"(d) : "h"(a), "h"(b), "f"(c));
  } else {
    asm("fma.rn.f32.bf16 %0, %1, %2, %3;" : "=f"(d) : "h"(a), "h"(b), "f"(c));
  }
  return d;
}

// acc + sum of squares of the vector's elements, on two chains (even and odd
// elements) so that consecutive FMAs do not wait on each other.
template <typename T>
__device__ __forceinline__ float2 sumsq_vec(uint4 v, float2 acc) {
  if constexpr (sizeof(T) == 4) {
    acc.x = fmaf(__uint_as_float(v.x), __uint_as_float(v.x), acc.x);
    acc.y = fmaf(__uint_as_float(v.y), __uint_as_float(v.y), acc.y);
    acc.x = fmaf(__uint_as_float(v.z), __uint_as_float(v.z), acc.x);
    acc.y = fmaf(__uint_as_float(v.w), __uint_as_float(v.w), acc.y);
  } else {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint16_t lo = static_cast<uint16_t>(w[i]), hi = static_cast<uint16_t>(w[i] >> 16);
      acc.x = fma_mixed<T>(lo, lo, acc.x);
      acc.y = fma_mixed<T>(hi, hi, acc.y);
    }
  }
  return acc;
}

// The vector x * gamma * scale, rounded once to T.
template <typename T>
__device__ __forceinline__ uint4 scale_gamma_vec(uint4 x, uint4 g, float scale) {
  const uint64_t s2 = f2_splat(scale);
  const uint32_t xw[4] = {x.x, x.y, x.z, x.w}, gw[4] = {g.x, g.y, g.z, g.w};
  uint32_t out[4];
  if constexpr (sizeof(T) == 4) {
    // fp32 elements: x * gamma on pairs, then the scale
    const uint64_t p0 = f2_mul(f2_pack(__uint_as_float(xw[0]), __uint_as_float(xw[1])),
                               f2_pack(__uint_as_float(gw[0]), __uint_as_float(gw[1])));
    const uint64_t p1 = f2_mul(f2_pack(__uint_as_float(xw[2]), __uint_as_float(xw[3])),
                               f2_pack(__uint_as_float(gw[2]), __uint_as_float(gw[3])));
    const float2 a = f2_unpack(f2_mul(p0, s2)), b = f2_unpack(f2_mul(p1, s2));
    return make_uint4(__float_as_uint(a.x), __float_as_uint(a.y), __float_as_uint(b.x), __float_as_uint(b.y));
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float plo = fma_mixed<T>(static_cast<uint16_t>(xw[i]), static_cast<uint16_t>(gw[i]), -0.0f);
      const float phi = fma_mixed<T>(static_cast<uint16_t>(xw[i] >> 16), static_cast<uint16_t>(gw[i] >> 16), -0.0f);
      const float2 y = f2_unpack(f2_mul(f2_pack(plo, phi), s2));
      out[i] = RowVec<T>::from_f2(y.x, y.y);
    }
    return make_uint4(out[0], out[1], out[2], out[3]);
  }
}

// (max, sum of exp) over the 32 lanes of a warp: the maximum first, then each
// lane's sum rescaled to it by exp(m_lane - M). A lane with no elements has
// m = -inf and s = 0.
__device__ __forceinline__ float2 warp_max_sum(float m, float s) {
  float M = m;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
  float t = m == -INFINITY ? 0.0f : s * ex2_ftz((m - M) * kRowLog2e);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) t += __shfl_xor_sync(0xffffffffu, t, off);
  return make_float2(M, t);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

}  // namespace kf
