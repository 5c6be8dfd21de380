// Device-side building blocks shared by the sm_100a kernels: shared-memory
// addressing, mbarrier waits with a time limit, TMA tile loads and the
// tcgen05 (5th-generation tensor core + TMEM) instructions, all as inline PTX.
//
// Every wait on a barrier is bounded. A wait that exceeds KF_WAIT_LIMIT_NS
// records KF_ERR_TIMEOUT (plus a site code) in the per-device status word and
// raises the CTA's abort flag, so the other warp roles leave their loops and
// the CTA can release TMEM and exit instead of spinning forever.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernelo_b200.h"

#ifndef KF_WAIT_LIMIT_NS
#define KF_WAIT_LIMIT_NS 2000000000ull  // 2 s: far above any legitimate wait
#endif

namespace kf {

// ---------------------------------------------------------------- types
template <typename T> struct DType;
template <> struct DType<__half> { static constexpr int code = KF_FP16; };
template <> struct DType<__nv_bfloat16> { static constexpr int code = KF_BF16; };
template <> struct DType<float> { static constexpr int code = KF_FP32; };

__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f32(float v) { return v; }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }

// ---------------------------------------------------------------- status
// Site codes stored above the status code so a timeout names its wait.
enum WaitSite : int {
  SITE_TMA_EMPTY = 1,
  SITE_MMA_FULL = 2,
  SITE_MMA_TMEM_EMPTY = 3,
  SITE_EPI_TMEM_FULL = 4,
  SITE_DRAIN = 5,
  SITE_SELFTEST = 6,
  SITE_PEER_BARRIER = 7,
};

__device__ __forceinline__ void record_status(int* status, int code, int site) {
  if (status != nullptr) atomicCAS(status, 0, code | (site << 8));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- smem / mbarrier
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

// Waits for the phase with the given parity to complete. Returns false when
// the CTA's abort flag was raised or the time limit passed (which raises it).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          int* status, int site,
                                          uint64_t limit_ns = KF_WAIT_LIMIT_NS) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  for (uint32_t spin = 1;; ++spin) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((spin & 7u) == 0) {
      if (abort_flag != nullptr && *abort_flag) return false;
      if (global_timer_ns() - start > limit_ns) {
        record_status(status, KF_ERR_TIMEOUT, site);
        if (abort_flag != nullptr) *abort_flag = 1;
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------- bulk copies
// Untiled bulk copy of `bytes` (a multiple of 16; both addresses 16-byte
// aligned) from global memory into this CTA's shared memory, completing as
// transaction bytes on `bar`.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(dst),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
      : "memory");
}

// Orders this thread's earlier generic-proxy shared-memory accesses (and what
// a barrier made visible to it) before its following bulk copies.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- TMA
// 2-D tiled bulk tensor load into this CTA's shared memory; completion is
// signalled on `bar` as transaction bytes. x is the innermost coordinate.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t dst_slot_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   dst_slot_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] x B[smem desc], kind::f16 (fp16/bf16 in, fp32 accumulate).
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// The same with kind::tf32 (32-bit containers read as TF32, fp32 accumulate):
// the fp32 GEMM's split operands, whose parts are already TF32 values.
__device__ __forceinline__ void tc_mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when every tcgen05.mma issued so far by this thread completes.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}

// Each lane reads 16 consecutive 32-bit columns of TMEM lane (base lane + laneid).
__device__ __forceinline__ void tmem_ld_16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32"
      " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------- clusters / CTA pairs
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Every thread of every CTA in the cluster arrives and waits.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Address, in the cluster's shared window, of this CTA's `addr` in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

// Arrive on an mbarrier that may live in another CTA of the cluster.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

// TMA tile load issued by either CTA of an MMA pair; the transaction bytes are
// counted on `bar` (a cluster address: the leader CTA's barrier).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                                 int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// tcgen05 for a CTA pair (M = 256 across two SMs): TMEM is allocated and freed
// collectively by one warp of each CTA; only the leader issues MMAs.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_slot_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   dst_slot_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_mma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                                uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tc_mma_tf32_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                                 uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on the barrier at this offset in every CTA of `cta_mask` when the
// pair's MMAs issued so far complete.
__device__ __forceinline__ void tc_commit_pair_to(uint32_t bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(bar),
      "h"(cta_mask)
      : "memory");
}
__device__ __forceinline__ void tc_commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

// Shared-memory matrix descriptor (sm_100 format): start address, leading and
// stride byte offsets (16-byte units), descriptor version 1, 128-byte swizzle.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr, uint32_t lbo_bytes,
                                                    uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;  // version (Blackwell)
  d |= 2ull << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor with fp32 accumulation, for kind::f16 (fmt 0 = fp16,
// 1 = bf16) and kind::tf32 (fmt 2 = tf32), which share the layout.
// *_mn: operand is MN-major in shared memory.
__host__ __device__ constexpr uint32_t instr_desc_f16(uint32_t fmt, uint32_t a_mn, uint32_t b_mn,
                                                      uint32_t m, uint32_t n) {
  return (1u << 4)            // D format: f32
         | (fmt << 7)         // A format
         | (fmt << 10)        // B format
         | (a_mn << 15)       // A major
         | (b_mn << 16)       // B major
         | ((n >> 3) << 17)   // N / 8
         | ((m >> 4) << 24);  // M / 16
}

// ---------------------------------------------------------------- math
// GELU, written from its definition: exact form x * Phi(x) with
// Phi(x) = (1 + erf(x / sqrt(2))) / 2, and the tanh approximation
// 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))). CUDA's erff/tanhf are called.
// Hardware approximations (PTX ISA: relative error about 2^-22 / 2^-23;
// subnormal results flush to zero).
__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// The same without flushing: subnormal results are kept, which GELU's far
// negative tail needs (a bf16 output still resolves values near 1e-38).
__device__ __forceinline__ float ex2_sub(float x) {
  float y;
  asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_ftz(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Exact GELU, x * Phi(x), Phi(x) = erfc(-x / sqrt 2) / 2.
// erfc comes from the Chebyshev fit of W. H. Press et al., Numerical Recipes,
// 2nd ed., section 6.2 ("erfcc"): for z >= 0, with t = 1 / (1 + z/2),
//   erfc(z) = t * exp(-z^2 + P(t)),  P a degree-9 polynomial,
// with fractional error below 1.2e-7 over the whole range -- so Phi keeps its
// relative accuracy in the negative tail, where GELU is tiny. With the
// hardware reciprocal and exponential the result stays within about 2e-7
// relative (plus 2^-24 times |z^2| from rounding the exponent), far below
// half an ulp of an fp16 or bf16 output. For x >= 0, Phi = 1 - erfc(z) / 2.
__device__ __forceinline__ float gelu_erf(float x) {
  const float z = fabsf(x) * 0.70710678118654752440f;
  const float t = rcp_ftz(fmaf(0.5f, z, 1.0f));
  float p = fmaf(t, 0.17087277f, -0.82215223f);
  p = fmaf(t, p, 1.48851587f);
  p = fmaf(t, p, -1.13520398f);
  p = fmaf(t, p, 0.27886807f);
  p = fmaf(t, p, -0.18628806f);
  p = fmaf(t, p, 0.09678418f);
  p = fmaf(t, p, 0.37409196f);
  p = fmaf(t, p, 1.00002368f);
  p = fmaf(t, p, -1.26551223f);
  const float half_erfc = 0.5f * t * ex2_sub(fmaf(-z, z, p) * 1.4426950408889634f);
  return x * (x >= 0.0f ? 1.0f - half_erfc : half_erfc);
}

// tanh GELU, 0.5 x (1 + tanh(u)) with u = sqrt(2/pi) (x + 0.044715 x^3),
// through the identity 1 + tanh(u) = 2 / (1 + exp(-2u)). With e = exp(-2|u|)
// in (0, 1]:
//   gelu = x / (1 + e)      for u >= 0,
//   gelu = x e / (1 + e)    for u < 0,
// which never overflows and keeps relative accuracy at both ends (no
// 1 + tanh cancellation for u << 0). The constants define the function
// (kernelforge/kernels/fused_linear.py).
__device__ __forceinline__ float gelu_tanh(float x) {
  const float u = 0.79788456080286535588f * fmaf(0.044715f * x, x * x, x);
  const float e = ex2_sub(fabsf(u) * (-2.0f * 1.4426950408889634f));
  const float r = rcp_ftz(1.0f + e);
  return x * (u >= 0.0f ? r : e * r);
}

// ---- packed fp32x2 arithmetic (sm_100: one instruction for two lanes)
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float2 f2_unpack(uint64_t v) {
  float a, b;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
  return make_float2(a, b);
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_splat(float a) { return f2_pack(a, a); }

// gelu_erf on two values: the same operations and roundings as gelu_erf,
// with the polynomial and the scalings done pairwise.
__device__ __forceinline__ float2 gelu_erf2(float2 x) {
  const float z0 = fabsf(x.x) * 0.70710678118654752440f;
  const float z1 = fabsf(x.y) * 0.70710678118654752440f;
  const float2 d = f2_unpack(f2_fma(f2_splat(0.5f), f2_pack(z0, z1), f2_splat(1.0f)));
  const uint64_t t = f2_pack(rcp_ftz(d.x), rcp_ftz(d.y));
  uint64_t p = f2_fma(t, f2_splat(0.17087277f), f2_splat(-0.82215223f));
  p = f2_fma(t, p, f2_splat(1.48851587f));
  p = f2_fma(t, p, f2_splat(-1.13520398f));
  p = f2_fma(t, p, f2_splat(0.27886807f));
  p = f2_fma(t, p, f2_splat(-0.18628806f));
  p = f2_fma(t, p, f2_splat(0.09678418f));
  p = f2_fma(t, p, f2_splat(0.37409196f));
  p = f2_fma(t, p, f2_splat(1.00002368f));
  p = f2_fma(t, p, f2_splat(-1.26551223f));
  const float2 pf = f2_unpack(p);
  const uint64_t e = f2_pack(ex2_sub(fmaf(-z0, z0, pf.x) * 1.4426950408889634f),
                             ex2_sub(fmaf(-z1, z1, pf.y) * 1.4426950408889634f));
  const float2 he = f2_unpack(f2_mul(f2_mul(f2_splat(0.5f), t), e));
  const float phi0 = x.x >= 0.0f ? 1.0f - he.x : he.x;
  const float phi1 = x.y >= 0.0f ? 1.0f - he.y : he.y;
  return f2_unpack(f2_mul(f2_pack(x.x, x.y), f2_pack(phi0, phi1)));
}

// gelu_tanh on two values, pairwise where the arithmetic allows.
__device__ __forceinline__ float2 gelu_tanh2(float2 x) {
  const uint64_t xv = f2_pack(x.x, x.y);
  const uint64_t x2 = f2_mul(xv, xv);
  const uint64_t inner = f2_fma(f2_mul(f2_splat(0.044715f), xv), x2, xv);
  const float2 u = f2_unpack(f2_mul(f2_splat(0.79788456080286535588f), inner));
  const float e0 = ex2_sub(fabsf(u.x) * (-2.0f * 1.4426950408889634f));
  const float e1 = ex2_sub(fabsf(u.y) * (-2.0f * 1.4426950408889634f));
  const float2 den = f2_unpack(f2_add(f2_pack(e0, e1), f2_splat(1.0f)));
  const float r0 = rcp_ftz(den.x), r1 = rcp_ftz(den.y);
  return f2_unpack(f2_mul(xv, f2_pack(u.x >= 0.0f ? r0 : e0 * r0, u.y >= 0.0f ? r1 : e1 * r1)));
}

// The epilogue on two adjacent outputs.
template <int EPI>
__device__ __forceinline__ float2 apply_epilogue2(float2 acc, float2 bias) {
  if constexpr (EPI == KF_EPI_NONE) {
    return acc;
  } else {
    const float2 v = f2_unpack(f2_add(f2_pack(acc.x, acc.y), f2_pack(bias.x, bias.y)));
    if constexpr (EPI == KF_EPI_BIAS) {
      return v;
    } else if constexpr (EPI == KF_EPI_BIAS_GELU_TANH) {
      return gelu_tanh2(v);
    } else {
      return gelu_erf2(v);
    }
  }
}

template <int EPI>
__device__ __forceinline__ float apply_epilogue(float acc, float bias) {
  if constexpr (EPI == KF_EPI_NONE) {
    return acc;
  } else if constexpr (EPI == KF_EPI_BIAS) {
    return acc + bias;
  } else if constexpr (EPI == KF_EPI_BIAS_GELU_TANH) {
    return gelu_tanh(acc + bias);
  } else {
    return gelu_erf(acc + bias);
  }
}

// ---------------------------------------------------------------- programmatic dependent launch
// Lets the next grid on the stream (when launched with programmatic stream
// serialization) be scheduled before this one finishes.
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
// Waits until the grids this one depends on have completed and their memory
// operations are visible (returns at once for an ordinary launch).
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---------------------------------------------------------------- decode GEMV pieces
// Warp-level m16n8k16 tensor-core product with fp32 accumulation (the decode
// GEMVs' contraction: 16 weight rows against 8 rows of x).
template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  if constexpr (DType<T>::code == KF_BF16) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

// A 16-byte vector of x (read-only for the kernel's lifetime, re-read by many
// warps): kept in L1 ahead of streaming lines.
__device__ __forceinline__ uint4 load_x(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::evict_last.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// The same from L2, bypassing L1: for a grid launched as a programmatic
// dependent, whose x is written by the previous grid during this grid's
// lifetime (the non-coherent path above may then return stale lines).
__device__ __forceinline__ uint4 load_x_l2(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

}  // namespace kf
