// Persistent row softmax / RMSNorm that streams rows through shared memory
// with bulk copies (sm_100a).
//
// A CTA holds NG row groups of G warps; each group is one "worker" that takes
// rows worker, worker + W, worker + 2W, ... (W = workers in the grid). Every
// group owns K shared-memory slots of one row each and keeps them full:
//   * its leader thread issues a cp.async.bulk of the row's 16-byte-aligned
//     interior into a slot, completing on the slot's mbarrier (K rows ahead);
//   * the group waits for the slot, copies the row into registers (a thread
//     holds NV 16-byte vectors), and the leader at once refills the slot with
//     the row K steps ahead -- so loads stay in flight while the row is
//     reduced (warp shuffles; shared memory and a named barrier across the
//     group's warps), normalised from registers and written with 16-byte
//     streaming stores.
// Each row is read from HBM once and written once. Scalar head/tail elements
// (rows that do not start on a 16-byte boundary, e.g. 4097 fp16 columns) are
// read directly. RMSNorm's gamma is staged in shared memory once per CTA.
// Since a slot only ever carries its own group's rows, no cross-group
// release barrier is needed.
//
// Every wait is bounded; a timeout raises the CTA's abort flag and records
// KF_ERR_TIMEOUT in the device status word. A group decides to stop as a
// whole (warp vote, then a barrier reduction across its warps), and its
// leader waits (bounded) for the copies it still has in flight before the
// group leaves, so no copy lands in released shared memory and no warp is left
// at a named barrier its partners skipped.
//
// Semantics follow kernelforge/kernels/softmax.py:31-58 and
// kernelforge/kernels/rmsnorm.py:41-72 (fp32 statistics, one rounding).
#include "kf_common.cuh"
#include "kf_internal.h"
#include "rows_math.cuh"

namespace kf {
namespace {

constexpr int OP_SOFTMAX = 0;
constexpr int OP_RMSNORM = 1;
constexpr int MAX_WARPS = 16;  // per CTA
constexpr int MAX_SLOTS_PER_GROUP = 8;
constexpr int STREAM_THREADS = 32 * MAX_WARPS;
// Shared memory besides the slots and gamma: alignment slack, barriers are
// counted per slot, group partials [16][16] float2, abort flag.
constexpr int STREAM_FIXED_SMEM = 128 + 8 * MAX_WARPS * MAX_WARPS + 16;
// Bytes of shared memory on one SM, and what the runtime reserves per CTA.
constexpr int SM100_SMEM_PER_SM = 233472;
constexpr int SMEM_RESERVED_PER_CTA = 1024;

struct StreamParams {
  const void* x;
  long long sx;
  const void* gamma;
  void* y;
  long long sy;
  long long rows;
  int cols;
  float eps;
  float inv_cols;
  int G;   // warps per row group
  int NG;  // row groups per CTA
  int K;   // slots per group
  uint32_t stage_bytes;
  uint32_t gamma_bytes;  // 0: gamma read from global memory
  int* status;
};

__device__ __forceinline__ void group_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Named barrier that also ANDs a predicate over the participating threads.
__device__ __forceinline__ bool group_bar_and(int id, int threads, bool pred) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(out)
      : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(threads)
      : "memory");
  return out != 0;
}

template <typename T>
__device__ __forceinline__ int row_head(const T* row, int cols) {
  const uint32_t addr = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(row));
  const int head = static_cast<int>(((16u - (addr & 15u)) & 15u) / sizeof(T));
  return head < cols ? head : cols;
}

// Leader: arm `bar` for row `row` and copy its interior into `slot`.
template <typename T>
__device__ __forceinline__ void issue_row(const StreamParams& p, long long row, uint8_t* slot,
                                          uint32_t bar) {
  constexpr int VE = RowVec<T>::VE;
  const T* xr = static_cast<const T*>(p.x) + row * p.sx;
  const int head = row_head(xr, p.cols);
  const uint32_t bytes = static_cast<uint32_t>((p.cols - head) / VE) * 16u;
  if (bytes > 0) {
    mbar_arrive_expect_tx(bar, bytes);
    bulk_load(smem_u32(slot), xr + head, bytes, bar);
  } else {
    mbar_arrive(bar);
  }
}

template <int NV>
constexpr int stream_min_blocks() {
  // Two 512-thread CTAs per SM need <= 64 registers a thread, which holds
  // only up to two vectors a thread without spilling.
  return NV <= 2 ? 2 : 1;
}

template <typename T, int NV, int OP>
__global__ void __launch_bounds__(STREAM_THREADS, stream_min_blocks<NV>())
    rows_stream_kernel(const StreamParams p) {
  constexpr int VE = RowVec<T>::VE;
  // Softmax keeps exp(x - m_thread) in registers when that fits; wider rows
  // evaluate it again in the output pass (same value either way).
  constexpr bool KEEP_EV = OP == OP_SOFTMAX && NV * VE <= 32;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) &
                                             ~static_cast<uintptr_t>(127));
  const int G = p.G, NG = p.NG, K = p.K;
  const int nslots = NG * K;
  uint8_t* ring = smem;
  T* gamma_s = reinterpret_cast<T*>(ring + static_cast<size_t>(nslots) * p.stage_bytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(gamma_s) + p.gamma_bytes);
  float2* parts = reinterpret_cast<float2*>(bars + nslots);  // [NG][MAX_WARPS]
  volatile int* abort_flag = reinterpret_cast<volatile int*>(parts + MAX_WARPS * MAX_WARPS);

  if (threadIdx.x == 0) {
    for (int s = 0; s < nslots; ++s) mbar_init(smem_u32(bars + s), 1);
    *abort_flag = 0;
    mbar_init_fence();
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = warp / G, wig = warp % G;
  const int tg = wig * 32 + lane;  // thread index within the row group
  const int TG = G * 32;
  const bool leader = tg == 0;
  const long long W = static_cast<long long>(gridDim.x) * NG;
  const long long ahead = W * K;
  uint8_t* my_ring = ring + static_cast<size_t>(g) * K * p.stage_bytes;
  const uint32_t my_bar = smem_u32(bars + g * K);
  float2* my_parts = parts + g * MAX_WARPS;

  long long row = static_cast<long long>(blockIdx.x) * NG + g;
  // The first copies go out before anything else, gamma staging included.
  if (leader) {
    long long r = row;
    for (int u = 0; u < K && r < p.rows; ++u, r += W)
      issue_row<T>(p, r, my_ring + static_cast<size_t>(u) * p.stage_bytes, my_bar + 8u * u);
  }
  if constexpr (OP == OP_RMSNORM) {
    if (p.gamma_bytes != 0) {  // every row of this CTA reads gamma: stage it once
      const T* gg = static_cast<const T*>(p.gamma);
      for (int i = threadIdx.x; i < p.cols; i += blockDim.x) gamma_s[i] = gg[i];
    }
    __syncthreads();
  }

  // Scalar head/tail elements of a row (outside its 16-byte-aligned interior),
  // loaded one row ahead so their latency hides behind the current row.
  auto edges = [&](long long r, float& h, float& t) {
    h = 0.0f;
    t = 0.0f;
    if (r < p.rows) {
      const T* xr = static_cast<const T*>(p.x) + r * p.sx;
      const int hd = row_head(xr, p.cols);
      const int nv = (p.cols - hd) / VE;
      if (tg < hd) h = to_f32(xr[tg]);
      if (tg < p.cols - hd - nv * VE) t = to_f32(xr[hd + nv * VE + tg]);
    }
  };
  float next_h, next_t;
  edges(row, next_h, next_t);

  int slot = 0;
  uint32_t phase = 0;
  for (; row < p.rows; row += W) {
    const T* xr = static_cast<const T*>(p.x) + row * p.sx;
    T* yr = static_cast<T*>(p.y) + row * p.sy;
    const int head = row_head(xr, p.cols);
    const int nvec = (p.cols - head) / VE;
    const int tail = p.cols - head - nvec * VE;
    const bool has_head = tg < head, has_tail = tg < tail;
    const int tail_idx = head + nvec * VE + tg;
    const float xh = next_h, xt = next_t;
    edges(row + W, next_h, next_t);

    uint8_t* slot_ptr = my_ring + static_cast<size_t>(slot) * p.stage_bytes;
    bool ok = mbar_wait(my_bar + 8u * slot, phase, abort_flag, p.status, SITE_MMA_FULL);
    // Read the slot even when the wait failed (a stale read cannot fault); the
    // values are discarded below.
    const uint4* sv = reinterpret_cast<const uint4*>(slot_ptr);
    uint4 raw[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int v = tg + j * TG;
      if (v < nvec) raw[j] = sv[v];
    }
    ok = __all_sync(0xffffffffu, ok);
    if (G > 1) {
      ok = group_bar_and(1 + g, TG, ok);  // also: every warp has read the slot
    } else {
      __syncwarp();
    }
    if (!ok) {
      if (leader) {  // let this group's copies still in flight land
        long long r = row;
        int s = slot;
        uint32_t ph = phase;
        for (int u = 0; u < K && r < p.rows; ++u, r += W) {
          mbar_wait(my_bar + 8u * s, ph, nullptr, p.status, SITE_DRAIN, 100000000ull);
          if (++s == K) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      break;
    }
    if (leader && row + ahead < p.rows) {
      fence_proxy_async_smem();
      issue_row<T>(p, row + ahead, slot_ptr, my_bar + 8u * slot);
    }
    if (++slot == K) {
      slot = 0;
      phase ^= 1u;
    }

    // ---- this thread's statistic
    float ev[KEEP_EV ? NV * VE : 1];
    float m_thr = -INFINITY, eh = 0.0f, et = 0.0f;
    float2 part;
    if constexpr (OP == OP_SOFTMAX) {
      uint4 mv = RowVec<T>::lowest();
#pragma unroll
      for (int j = 0; j < NV; ++j)
        if (tg + j * TG < nvec) mv = vmax<T>(mv, raw[j]);
      m_thr = hmax<T>(mv);
      if (has_head) m_thr = fmaxf(m_thr, xh);
      if (has_tail) m_thr = fmaxf(m_thr, xt);
      float s = 0.0f;
      if (m_thr != -INFINITY) {
        const float mb = m_thr * kRowLog2e;
#pragma unroll
        for (int j = 0; j < NV; ++j) {
          if (tg + j * TG < nvec) {
            float f[VE];
            to_floats<T>(raw[j], f);
#pragma unroll
            for (int k = 0; k < VE; ++k) {
              const float t = ex2_ftz(fmaf(f[k], kRowLog2e, -mb));
              if constexpr (KEEP_EV) ev[j * VE + k] = t;
              s += t;
            }
          }
        }
        if (has_head) s += (eh = ex2_ftz(fmaf(xh, kRowLog2e, -mb)));
        if (has_tail) s += (et = ex2_ftz(fmaf(xt, kRowLog2e, -mb)));
      }
      part = warp_max_sum(m_thr, s);
    } else {
      float ss = 0.0f;
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        if (tg + j * TG < nvec) {
          float f[VE];
          to_floats<T>(raw[j], f);
#pragma unroll
          for (int k = 0; k < VE; ++k) ss = fmaf(f[k], f[k], ss);
        }
      }
      if (has_head) ss = fmaf(xh, xh, ss);
      if (has_tail) ss = fmaf(xt, xt, ss);
      part = make_float2(warp_sum(ss), 0.0f);
    }

    // ---- across the group's warps: each warp combines all G partials lane-parallel
    if (G > 1) {
      if (lane == 0) my_parts[wig] = part;
      group_bar_sync(1 + g, TG);
      // Single buffer: the next write comes after the next iteration's
      // barrier, which every warp reaches only after reading this one.
      const float2 o = lane < G ? my_parts[lane] : make_float2(-INFINITY, 0.0f);
      if constexpr (OP == OP_SOFTMAX) {
        part = warp_max_sum(o.x, o.y);
      } else {
        part = make_float2(warp_sum(lane < G ? o.x : 0.0f), 0.0f);
      }
    }

    // ---- normalise from registers and write
    uint4* yv = reinterpret_cast<uint4*>(yr + head);
    if constexpr (OP == OP_SOFTMAX) {
      // exp(x - M) / S = exp(x - m_thr) * (exp(m_thr - M) / S)
      const float factor =
          m_thr == -INFINITY ? 0.0f : ex2_ftz((m_thr - part.x) * kRowLog2e) / part.y;
      const float mb = m_thr * kRowLog2e;
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int v = tg + j * TG;
        if (v < nvec) {
          float o[VE];
          if constexpr (KEEP_EV) {
#pragma unroll
            for (int k = 0; k < VE; ++k) o[k] = ev[j * VE + k] * factor;
          } else {
            to_floats<T>(raw[j], o);
#pragma unroll
            for (int k = 0; k < VE; ++k) o[k] = ex2_ftz(fmaf(o[k], kRowLog2e, -mb)) * factor;
          }
          __stcs(yv + v, from_floats<T>(o));
        }
      }
      if (has_head) yr[tg] = from_f32<T>(eh * factor);
      if (has_tail) yr[tail_idx] = from_f32<T>(et * factor);
    } else {
      const float scale = rsqrtf(part.x * p.inv_cols + p.eps);
      const T* gsrc = p.gamma_bytes != 0 ? gamma_s : static_cast<const T*>(p.gamma);
      const bool gvec = head == 0 && (reinterpret_cast<uintptr_t>(gsrc) & 15u) == 0;
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int v = tg + j * TG;
        if (v < nvec) {
          float f[VE], gf[VE];
          to_floats<T>(raw[j], f);
          if (gvec) {
            to_floats<T>(reinterpret_cast<const uint4*>(gsrc)[v], gf);
          } else {
#pragma unroll
            for (int k = 0; k < VE; ++k) gf[k] = to_f32(gsrc[head + v * VE + k]);
          }
#pragma unroll
          for (int k = 0; k < VE; ++k) f[k] = f[k] * scale * gf[k];
          __stcs(yv + v, from_floats<T>(f));
        }
      }
      if (has_head) yr[tg] = from_f32<T>(xh * scale * to_f32(gsrc[tg]));
      if (has_tail) yr[tail_idx] = from_f32<T>(xt * scale * to_f32(gsrc[tail_idx]));
    }
  }
}

size_t stream_smem(const StreamParams& p) {
  return STREAM_FIXED_SMEM + static_cast<size_t>(p.NG) * p.K * (p.stage_bytes + 8) +
         p.gamma_bytes;
}

int vectors_per_thread(int64_t cols, int elem, int warps) {
  const int64_t nvec = cols * elem / 16;
  const int64_t n = ceil_div(nvec, 32LL * warps);
  return static_cast<int>(n < 1 ? 1 : n);
}

template <typename T, int NV, int OP>
int launch_stream_nv(StreamParams p, const kf_rows_config& cfg, const DeviceInfo& dev,
                     cudaStream_t stream) {
  auto fn = rows_stream_kernel<T, NV, OP>;
  const int threads = 32 * p.G * p.NG;
  // CTAs per SM the registers allow, then the shared memory each may take.
  int occ = 0;
  cudaError_t err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, threads, 0);
  if (err != cudaSuccess) return cuda_error(err, "occupancy(row stream)");
  if (occ < 1) return set_error(KF_ERR_INVALID_CONFIG, "streaming row kernel cannot launch");
  if (occ > 2) occ = 2;
  const int64_t fixed = STREAM_FIXED_SMEM + p.gamma_bytes;
  const int64_t per_slot = p.stage_bytes + 8;
  auto slots_at = [&](int ctas) {
    int64_t budget = SM100_SMEM_PER_SM / ctas - SMEM_RESERVED_PER_CTA;
    if (budget > dev.max_smem_optin) budget = dev.max_smem_optin;
    const int64_t k = (budget - fixed) / (per_slot * p.NG);
    return static_cast<int>(k > MAX_SLOTS_PER_GROUP ? MAX_SLOTS_PER_GROUP : k);
  };
  // Two CTAs per SM when each can still keep two rows per group in flight
  // (or the slots asked for); otherwise one CTA with the whole shared memory.
  const int want = cfg.stages > 0 ? cfg.stages : 2;
  if (occ == 2 && slots_at(2) < want) occ = 1;
  int K = slots_at(occ);
  if (cfg.stages > 0) {
    if (cfg.stages > K)
      return set_error(KF_ERR_INVALID_CONFIG,
                       std::to_string(cfg.stages) + " row slots per group of " +
                           std::to_string(p.stage_bytes) + " bytes exceed shared memory");
    K = cfg.stages;
  }
  if (K < 1)
    return set_error(KF_ERR_INVALID_CONFIG,
                     std::to_string(p.NG) + " row groups with one " +
                         std::to_string(p.stage_bytes) + "-byte slot each exceed shared memory");
  p.K = K;
  const size_t smem = stream_smem(p);
  err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (err != cudaSuccess) return cuda_error(err, "cudaFuncSetAttribute(row stream)");
  int64_t grid = static_cast<int64_t>(dev.sm_count) * occ;
  const int64_t needed = ceil_div(p.rows, p.NG);
  if (grid > needed) grid = needed;
  fn<<<static_cast<unsigned>(grid), threads, smem, stream>>>(p);
  err = cudaGetLastError();
  if (err != cudaSuccess) return cuda_error(err, "launch(row stream)");
  return KF_OK;
}

template <typename T, int OP>
int launch_stream_typed(const RowsArgs& a, const kf_rows_config& cfg, const DeviceInfo& dev,
                        cudaStream_t stream) {
  StreamParams p{};
  p.x = a.x;
  p.sx = a.sx;
  p.gamma = a.gamma;
  p.y = a.y;
  p.sy = a.sy;
  p.rows = a.rows;
  p.cols = static_cast<int>(a.cols);
  p.eps = a.eps;
  p.inv_cols = 1.0f / static_cast<float>(a.cols);
  p.status = dev.status;
  p.G = cfg.num_warps;
  const int nv = vectors_per_thread(a.cols, sizeof(T), p.G);
  if (nv > 16)
    return set_error(KF_ERR_INVALID_CONFIG,
                     "register pressure: " + std::to_string(nv) +
                         " vectors per thread in the streaming kernel; use more warps per row");
  const int64_t row_bytes = a.cols * static_cast<int64_t>(sizeof(T));
  p.stage_bytes = static_cast<uint32_t>(ceil_div(row_bytes / 16 * 16, 128) * 128);
  if (p.stage_bytes == 0) p.stage_bytes = 128;
  const int ng = cfg.row_groups > 0 ? cfg.row_groups : MAX_WARPS / p.G;
  if (ng * p.G > MAX_WARPS)
    return set_error(KF_ERR_INVALID_CONFIG, "row_groups x num_warps must be at most 16 warps");
  p.NG = ng;
  // Stage gamma in shared memory when a slot per group still fits beside it.
  const int64_t gamma_bytes = OP == OP_RMSNORM ? ceil_div(row_bytes, 128) * 128 : 0;
  p.gamma_bytes = (gamma_bytes > 0 && STREAM_FIXED_SMEM + gamma_bytes +
                                              int64_t(ng) * (p.stage_bytes + 8) <=
                                          dev.max_smem_optin)
                      ? static_cast<uint32_t>(gamma_bytes)
                      : 0u;
  if (nv <= 1) return launch_stream_nv<T, 1, OP>(p, cfg, dev, stream);
  if (nv <= 2) return launch_stream_nv<T, 2, OP>(p, cfg, dev, stream);
  if (nv <= 4) return launch_stream_nv<T, 4, OP>(p, cfg, dev, stream);
  if (nv <= 8) return launch_stream_nv<T, 8, OP>(p, cfg, dev, stream);
  return launch_stream_nv<T, 16, OP>(p, cfg, dev, stream);
}

}  // namespace

bool rows_stream_supported(const RowsArgs& a, int max_smem_optin, std::string* why) {
  const int elem = a.dtype == KF_FP32 ? 4 : 2;
  const uintptr_t xa = reinterpret_cast<uintptr_t>(a.x), ya = reinterpret_cast<uintptr_t>(a.y);
  // The output is written with the input row's head/vector/tail split, so x
  // and y rows must sit at the same 16-byte phase.
  if ((xa % elem) != 0 || (xa & 15u) != (ya & 15u) ||
      ((a.sx * elem) & 15) != ((a.sy * elem) & 15)) {
    if (why) *why = "x and y rows are not at the same 16-byte phase";
    return false;
  }
  const int64_t slot = ceil_div(a.cols * elem / 16 * 16, 128) * 128;
  if (STREAM_FIXED_SMEM + slot + 8 > max_smem_optin) {
    if (why) *why = "a row does not fit one shared-memory slot";
    return false;
  }
  if (vectors_per_thread(a.cols, elem, MAX_WARPS) > 16) {
    if (why) *why = "a row needs more than 16 vectors per thread at 16 warps";
    return false;
  }
  return true;
}

int stream_default_warps(int64_t cols, int elem) {
  // The fewest warps that hold the row at up to 16 vectors a thread (more
  // groups per CTA means more rows in flight), as a power of two so that row
  // groups tile the CTA's 16 warps.
  const int64_t nvec = cols * elem / 16;
  int64_t warps = ceil_div(nvec, 32 * 16);
  if (warps > MAX_WARPS) warps = MAX_WARPS;
  int p2 = 1;
  while (p2 < warps) p2 <<= 1;
  return p2;
}

int launch_rows_stream(const RowsArgs& a, const kf_rows_config& cfg, const DeviceInfo& dev,
                       cudaStream_t stream) {
  if (cfg.num_warps < 1 || cfg.num_warps > MAX_WARPS)
    return set_error(KF_ERR_INVALID_CONFIG, "the streaming row kernel takes 1..16 warps per row");
  if (cfg.row_groups < 0 || cfg.stages < 0)
    return set_error(KF_ERR_INVALID_CONFIG, "row_groups and stages must be >= 0");
  if (a.cols > INT32_MAX) return set_error(KF_ERR_UNSUPPORTED, "row too wide");
  std::string why;
  if (!rows_stream_supported(a, dev.max_smem_optin, &why))
    return set_error(KF_ERR_UNALIGNED, "streaming row kernel: " + why);
  if (a.rows == 0 || a.cols == 0) return KF_OK;
  if (a.op == OP_SOFTMAX) {
    switch (a.dtype) {
      case KF_FP16: return launch_stream_typed<__half, OP_SOFTMAX>(a, cfg, dev, stream);
      case KF_BF16: return launch_stream_typed<__nv_bfloat16, OP_SOFTMAX>(a, cfg, dev, stream);
      case KF_FP32: return launch_stream_typed<float, OP_SOFTMAX>(a, cfg, dev, stream);
    }
  } else {
    switch (a.dtype) {
      case KF_FP16: return launch_stream_typed<__half, OP_RMSNORM>(a, cfg, dev, stream);
      case KF_BF16: return launch_stream_typed<__nv_bfloat16, OP_RMSNORM>(a, cfg, dev, stream);
      case KF_FP32: return launch_stream_typed<float, OP_RMSNORM>(a, cfg, dev, stream);
    }
  }
  return set_error(KF_ERR_INVALID_ARGUMENT, "unknown dtype code");
}

}  // namespace kf
