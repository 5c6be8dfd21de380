// Row-wise softmax and RMSNorm for sm_100a: one read of x, one write of y.
//
// A row is owned by one CTA, or by a thread-block cluster of `cluster` CTAs
// when it is too wide for one CTA's registers (softmax over 32000 fp32 columns
// is 128 KB per row). Each thread loads its share of the row with 128-bit
// vector loads straight into registers, keeps it there while the row's
// statistic is reduced (warp shuffles, then shared memory across warps, then
// distributed shared memory across the cluster), and writes the normalised
// values back with 128-bit stores. The row is never re-read from memory.
//
// Rows whose start is not 16-byte aligned (e.g. 4097 fp16 columns) are split
// into a scalar head, a vector body and a scalar tail, so every access stays
// inside the row. Softmax reduces (max, sum of exp) pairs in one pass: each
// thread sums exp(x - m_thread); a warp takes the maximum M first and rescales
// each lane's sum by exp(m_lane - M); warps and cluster CTAs combine the same
// way. The per-element arithmetic lives in rows_math.cuh.
//
// Reference semantics: kernelforge/kernels/softmax.py:31-58 (max-shifted exp,
// fp32 math, output rounded once) and kernelforge/kernels/rmsnorm.py:41-72,
// 130-143 (fp32 sum of squares, x * rsqrt(mean + eps) * gamma, one rounding).
// The reference kernels cap rows at 16384 columns (search.py:459); these do not.
#include <cooperative_groups.h>

#include "kf_common.cuh"
#include "kf_internal.h"
#include "rows_math.cuh"

namespace cg = cooperative_groups;

namespace kf {
namespace {

constexpr int OP_SOFTMAX = 0;
constexpr int OP_RMSNORM = 1;

struct RowsParams {
  const void* x;
  long long sx;
  const void* gamma;
  void* y;
  long long sy;
  long long rows;
  int cols;
  int rows_per_cta;
  float eps;
  float inv_cols;
};

template <typename T, int VE>
struct alignas(sizeof(T) * VE) Vec {
  T e[VE];
};

// 128-bit streaming accesses for 16-byte vectors (x is read once, y written
// once: evict-first); plain accesses for the scalar path.
template <typename V>
__device__ __forceinline__ V load_stream(const V* ptr) {
  if constexpr (sizeof(V) == 16) {
    const uint4 u = __ldcs(reinterpret_cast<const uint4*>(ptr));
    V out;
    memcpy(&out, &u, 16);
    return out;
  } else {
    return *ptr;
  }
}
template <typename V>
__device__ __forceinline__ V load_cached(const V* ptr) {
  if constexpr (sizeof(V) == 16) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(ptr));
    V out;
    memcpy(&out, &u, 16);
    return out;
  } else {
    return *ptr;
  }
}
template <typename V>
__device__ __forceinline__ void store_stream(V* ptr, const V& v) {
  if constexpr (sizeof(V) == 16) {
    uint4 u;
    memcpy(&u, &v, 16);
    __stcs(reinterpret_cast<uint4*>(ptr), u);
  } else {
    *ptr = v;
  }
}

template <int NV>
constexpr int max_threads_for() {
  return NV <= 4 ? 1024 : (NV <= 8 ? 512 : 256);
}

template <typename T, int VE>
__device__ __forceinline__ uint4 as_u4(const Vec<T, VE>& v) {
  static_assert(sizeof(Vec<T, VE>) == 16, "16-byte vectors only");
  return *reinterpret_cast<const uint4*>(&v);
}

// The VE elements of one loaded vector as fp32.
template <typename T, int VE>
__device__ __forceinline__ void vec_floats(const Vec<T, VE>& v, float* f) {
  if constexpr (VE > 1) {
    to_floats<T>(as_u4(v), f);
  } else {
    f[0] = to_f32(v.e[0]);
  }
}

template <typename T, int VE>
__device__ __forceinline__ Vec<T, VE> vec_from_floats(const float* f) {
  Vec<T, VE> o;
  if constexpr (VE > 1) {
    const uint4 u = from_floats<T>(f);
    memcpy(&o, &u, 16);
  } else {
    o.e[0] = from_f32<T>(f[0]);
  }
  return o;
}

template <typename T, int VE, int NV, int OP>
__global__ void __launch_bounds__(max_threads_for<NV>()) rows_kernel(const RowsParams p) {
  using V = Vec<T, VE>;
  cg::cluster_group cluster = cg::this_cluster();
  const unsigned crank = cluster.block_rank();
  const unsigned csize = cluster.num_blocks();
  const long long cluster_id = blockIdx.x / csize;
  const int nthreads = blockDim.x;
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int nwarps = (nthreads + 31) >> 5;
  const int g = static_cast<int>(crank) * nthreads + tid;  // thread index within the row
  const int G = static_cast<int>(csize) * nthreads;        // threads per row
  // Softmax keeps exp(x - m_thread) in registers when that fits; wider rows
  // evaluate it again in the output pass (same value either way).
  // (at most 16 values: more pushed the fp32 rows past 64 registers and
  // halved the resident warps, ncu: 4 CTAs of 128 threads per SM)
  constexpr bool KEEP_EV = OP == OP_SOFTMAX && NV * VE <= 16;

  __shared__ float2 warp_part[2][32];
  __shared__ float2 cta_part[2];  // read by the other CTAs of the cluster

  const T* gamma = static_cast<const T*>(p.gamma);

  for (int i = 0; i < p.rows_per_cta; ++i) {
    const long long row = cluster_id * p.rows_per_cta + i;
    if (row >= p.rows) break;  // uniform over the cluster
    const int par = i & 1;
    const T* xr = static_cast<const T*>(p.x) + row * p.sx;
    T* yr = static_cast<T*>(p.y) + row * p.sy;

    int head = 0;
    if (VE > 1) {
      const uint32_t addr = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(xr));
      head = static_cast<int>(((16u - (addr & 15u)) & 15u) / sizeof(T));
      if (head > p.cols) head = p.cols;
    }
    const int nvec = (p.cols - head) / VE;
    const int tail = p.cols - head - nvec * VE;
    const V* xv = reinterpret_cast<const V*>(xr + head);

    // ---- load: all vector loads issued before any use
    V raw[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int v = g + j * G;
      if (v < nvec) raw[j] = load_stream(xv + v);
    }
    const bool has_head = g < head;
    const bool has_tail = g < tail;
    const int tail_idx = head + nvec * VE + g;
    const float xh = has_head ? to_f32(xr[g]) : 0.0f;
    const float xt = has_tail ? to_f32(xr[tail_idx]) : 0.0f;

    // ---- per-thread partial, reduced over the warp
    float2 part;
    float ev[KEEP_EV ? NV * VE : 1];
    float eh = 0.0f, et = 0.0f, m_thr = -INFINITY;
    if constexpr (OP == OP_SOFTMAX) {
      if constexpr (VE > 1) {
        uint4 mv = RowVec<T>::lowest();
#pragma unroll
        for (int j = 0; j < NV; ++j)
          if (g + j * G < nvec) mv = vmax<T>(mv, as_u4(raw[j]));
        m_thr = hmax<T>(mv);
      } else {
#pragma unroll
        for (int j = 0; j < NV; ++j)
          if (g + j * G < nvec) m_thr = fmaxf(m_thr, to_f32(raw[j].e[0]));
      }
      if (has_head) m_thr = fmaxf(m_thr, xh);
      if (has_tail) m_thr = fmaxf(m_thr, xt);
      float s = 0.0f;
      if (m_thr != -INFINITY) {
        const float mb = m_thr * kRowLog2e;
#pragma unroll
        for (int j = 0; j < NV; ++j) {
          if (g + j * G < nvec) {
            float f[VE];
            vec_floats(raw[j], f);
#pragma unroll
            for (int e = 0; e < VE; ++e) {
              const float t = ex2_ftz(fmaf(f[e], kRowLog2e, -mb));
              if constexpr (KEEP_EV) ev[j * VE + e] = t;
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
      if constexpr (VE > 1) {
        // sm_100 mixed-precision FMA: the squares of 16-bit elements without
        // converting them first (rows_math.cuh: sumsq_vec)
        float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int j = 0; j < NV; ++j)
          if (g + j * G < nvec) acc = sumsq_vec<T>(as_u4(raw[j]), acc);
        ss = acc.x + acc.y;
      } else {
#pragma unroll
        for (int j = 0; j < NV; ++j)
          if (g + j * G < nvec) ss = fmaf(to_f32(raw[j].e[0]), to_f32(raw[j].e[0]), ss);
      }
      if (has_head) ss = fmaf(xh, xh, ss);
      if (has_tail) ss = fmaf(xt, xt, ss);
      part = make_float2(warp_sum(ss), 0.0f);
    }

    // ---- across warps, then across the cluster: lane-parallel combines
    float2 tot = part;
    if (nwarps > 1) {
      if (lane == 0) warp_part[par][warp] = part;
      __syncthreads();
      const float2 o = lane < nwarps ? warp_part[par][lane] : make_float2(-INFINITY, 0.0f);
      if constexpr (OP == OP_SOFTMAX) {
        tot = warp_max_sum(o.x, o.y);
      } else {
        tot = make_float2(warp_sum(lane < nwarps ? o.x : 0.0f), 0.0f);
      }
    }
    if (csize > 1) {
      if (tid == 0) cta_part[par] = tot;
      cluster.sync();
      const float2 o = lane < static_cast<int>(csize)
                           ? *cluster.map_shared_rank(&cta_part[par], static_cast<unsigned>(lane))
                           : make_float2(-INFINITY, 0.0f);
      if constexpr (OP == OP_SOFTMAX) {
        tot = warp_max_sum(o.x, o.y);
      } else {
        tot = make_float2(warp_sum(lane < static_cast<int>(csize) ? o.x : 0.0f), 0.0f);
      }
    }

    // ---- normalise and store
    V* yv = reinterpret_cast<V*>(yr + head);
    if constexpr (OP == OP_SOFTMAX) {
      // exp(x - M) / S = exp(x - m_thr) * (exp(m_thr - M) / S)
      const float factor =
          m_thr == -INFINITY ? 0.0f : ex2_ftz((m_thr - tot.x) * kRowLog2e) / tot.y;
      const float mb = m_thr * kRowLog2e;
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int v = g + j * G;
        if (v < nvec) {
          float o[VE];
          if constexpr (KEEP_EV) {
#pragma unroll
            for (int e = 0; e < VE; ++e) o[e] = ev[j * VE + e] * factor;
          } else {
            vec_floats(raw[j], o);
#pragma unroll
            for (int e = 0; e < VE; ++e) o[e] = ex2_ftz(fmaf(o[e], kRowLog2e, -mb)) * factor;
          }
          store_stream(yv + v, vec_from_floats<T, VE>(o));
        }
      }
      if (has_head) yr[g] = from_f32<T>(eh * factor);
      if (has_tail) yr[tail_idx] = from_f32<T>(et * factor);
    } else {
      const float scale = rsqrtf(tot.x * p.inv_cols + p.eps);
      const T* gb = gamma + head;
      const bool gamma_vec = VE > 1 && (reinterpret_cast<uintptr_t>(gb) & 15u) == 0;
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int v = g + j * G;
        if (v < nvec) {
          if constexpr (VE > 1) {
            if (gamma_vec) {
              // x * gamma exact (mixed-precision FMA), times the scale, one rounding
              const V gv = load_cached(reinterpret_cast<const V*>(gb) + v);
              const uint4 o = scale_gamma_vec<T>(as_u4(raw[j]), as_u4(gv), scale);
              V ov;
              memcpy(&ov, &o, 16);
              store_stream(yv + v, ov);
              continue;
            }
          }
          float f[VE], gf[VE];
          vec_floats(raw[j], f);
#pragma unroll
          for (int e = 0; e < VE; ++e) gf[e] = to_f32(gb[v * VE + e]);
#pragma unroll
          for (int e = 0; e < VE; ++e) f[e] = f[e] * gf[e] * scale;
          store_stream(yv + v, vec_from_floats<T, VE>(f));
        }
      }
      if (has_head) yr[g] = from_f32<T>(xh * to_f32(gamma[g]) * scale);
      if (has_tail) yr[tail_idx] = from_f32<T>(xt * to_f32(gamma[tail_idx]) * scale);
    }
  }
  // No CTA may leave while a peer could still read its cta_part.
  if (csize > 1) cluster.sync();
}

template <typename T, int VE, int NV, int OP>
int launch_one(const RowsParams& p, int threads, int cluster, long long clusters,
               cudaStream_t stream) {
  if (threads > max_threads_for<NV>())
    return set_error(KF_ERR_INVALID_CONFIG,
                     "register pressure: " + std::to_string(NV) + " vectors per thread allow at most " +
                         std::to_string(max_threads_for<NV>()) + " threads per CTA");
  cudaLaunchConfig_t lc{};
  lc.gridDim = dim3(static_cast<unsigned>(clusters * cluster));
  lc.blockDim = dim3(static_cast<unsigned>(threads));
  lc.dynamicSmemBytes = 0;
  lc.stream = stream;
  cudaLaunchAttribute attr[1];
  unsigned nattr = 0;
  if (cluster > 1) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(cluster);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    nattr = 1;
  }
  lc.attrs = attr;
  lc.numAttrs = nattr;
  cudaError_t err = cudaLaunchKernelEx(&lc, rows_kernel<T, VE, NV, OP>, p);
  if (err != cudaSuccess) return cuda_error(err, "launch(row kernel)");
  return KF_OK;
}

template <typename T, int VE, int OP>
int launch_nv(const RowsParams& p, int nv, int threads, int cluster, long long clusters,
              cudaStream_t stream) {
  if (nv <= 1) return launch_one<T, VE, 1, OP>(p, threads, cluster, clusters, stream);
  if (nv <= 2) return launch_one<T, VE, 2, OP>(p, threads, cluster, clusters, stream);
  if (nv <= 4) return launch_one<T, VE, 4, OP>(p, threads, cluster, clusters, stream);
  if (nv <= 8) return launch_one<T, VE, 8, OP>(p, threads, cluster, clusters, stream);
  if (nv <= 16) return launch_one<T, VE, 16, OP>(p, threads, cluster, clusters, stream);
  if (VE == 1 && nv <= 32) return launch_one<T, 1, 32, OP>(p, threads, cluster, clusters, stream);
  return set_error(KF_ERR_INVALID_CONFIG,
                   "register pressure: " + std::to_string(nv) +
                       " values per thread; use more warps or a larger cluster");
}

template <typename T, int OP>
int launch_typed(const RowsArgs& a, const kf_rows_config& cfg, cudaStream_t stream) {
  RowsParams p{};
  p.x = a.x;
  p.sx = a.sx;
  p.gamma = a.gamma;
  p.y = a.y;
  p.sy = a.sy;
  p.rows = a.rows;
  p.cols = static_cast<int>(a.cols);
  p.rows_per_cta = cfg.rows_per_cta;
  p.eps = a.eps;
  p.inv_cols = 1.0f / static_cast<float>(a.cols);
  constexpr int VEC = 16 / static_cast<int>(sizeof(T));
  // Vector path needs x and y rows to share their 16-byte phase.
  const uintptr_t xa = reinterpret_cast<uintptr_t>(a.x), ya = reinterpret_cast<uintptr_t>(a.y);
  const bool same_phase = (xa & 15u) == (ya & 15u) &&
                          ((a.sx * static_cast<long long>(sizeof(T))) & 15) ==
                              ((a.sy * static_cast<long long>(sizeof(T))) & 15) &&
                          (xa % sizeof(T)) == 0;
  const int threads = cfg.num_warps * 32;
  const long long per_row_threads = static_cast<long long>(threads) * cfg.cluster;
  const long long clusters = (a.rows + cfg.rows_per_cta - 1) / cfg.rows_per_cta;
  if (same_phase && a.cols >= VEC) {
    const long long nvec = a.cols / VEC;
    const int nv = static_cast<int>((nvec + per_row_threads - 1) / per_row_threads);
    return launch_nv<T, VEC, OP>(p, nv, threads, cfg.cluster, clusters, stream);
  }
  const int nv = static_cast<int>((a.cols + per_row_threads - 1) / per_row_threads);
  return launch_nv<T, 1, OP>(p, nv, threads, cfg.cluster, clusters, stream);
}

}  // namespace

kf_rows_config resolve_rows_config(const RowsArgs& a, const kf_rows_config* user,
                                   const DeviceInfo& dev) {
  kf_rows_config c{};
  if (user) c = *user;
  const int elem = a.dtype == KF_FP32 ? 4 : 2;
  if (c.kernel == KF_ROWS_AUTO) {
    // A field only one kernel has selects that kernel. Otherwise a softmax
    // with enough rows for every SM to stream several of them goes to the
    // persistent streaming kernel, which keeps loads in flight while rows are
    // reduced; the rest go to the register kernel, which can spread one row
    // over a cluster of SMs.
    const bool register_fields = c.rows_per_cta > 0 || c.cluster > 0 || c.num_warps > 16;
    const bool stream_fields = c.row_groups > 0 || c.stages > 0;
    // (the warp-per-row kernel has no fields of its own: it is chosen by width)
    if (register_fields != stream_fields) {
      c.kernel = register_fields ? KF_ROWS_REGISTER : KF_ROWS_STREAM;
    } else {
      // Measured on B200 (graph-timed, inputs beyond L2): softmax rows of up
      // to 2 KB stream (32768 x 1000 fp16: 0.78 of the copy bandwidth against
      // 0.70 in registers); rows up to 32 KB sit in registers at about eight
      // vectors per thread (2048 / 4096 / 8192 fp16 columns: 0.95 / 0.99 /
      // 0.98, against 0.80 / 0.80 / 0.87 streamed); wider rows stream again
      // (32000 fp16 columns: 0.99 streamed by 8-warp groups against 0.57 in
      // registers at 16 vectors a thread).
      // RMSNorm's lighter arithmetic runs as fast in the register kernel.
      const long long nvec_row = ceil_div(a.cols * elem, 16LL);
      const int warps = c.num_warps > 0 ? c.num_warps : stream_default_warps(a.cols, elem);
      const long long per_thread = ceil_div(nvec_row, 32LL * warps);
      const bool stream_ok = a.op == 0 && a.rows >= 2LL * dev.sm_count && per_thread <= 16 &&
                             rows_stream_supported(a, dev.max_smem_optin, nullptr);
      const bool narrow = nvec_row <= SOFTMAX_STREAM_MAX_VECTORS;
      const bool in_registers = nvec_row <= SOFTMAX_REGISTER_MAX_VECTORS;
      c.kernel = stream_ok && (narrow || !in_registers) ? KF_ROWS_STREAM : KF_ROWS_REGISTER;
      // Narrow rows on the 16-byte grid, either operation: a warp per row, no
      // shared memory. The streaming kernel is issue-bound on its per-row
      // machinery there (ncu: 67 % issue-active at 1000 fp16 columns), and
      // one CTA per row leaves few loads in flight. Measured on B200
      // (graph-timed, inputs beyond L2): softmax 32768 x 1000 fp16 1.05 of
      // the copy bandwidth against 0.81 streamed; RMSNorm 16384 x 1024 fp16
      // 1.09 against 0.87 in registers. RMSNorm keeps the gain up to 4 KB
      // rows (16384 x 2048 fp16 1.09 against 0.96; 16384 x 1024 fp32 1.20
      // against 0.91); softmax does not (32768 x 2048 fp16 0.85 against 0.96
      // in registers), its exponentials being the heavier per-lane work.
      const long long warp_max = a.op == 1 ? ROWS_WARP_RMSNORM_MAX_VECTORS : ROWS_WARP_MAX_VECTORS;
      if (nvec_row <= warp_max && a.rows >= 2LL * dev.sm_count && rows_warp_supported(a, nullptr))
        c.kernel = KF_ROWS_WARP;
      // Two slots per row group leave room for two CTAs per SM, which beats
      // deeper slots on narrow rows (25.8 against 27.6 us at 1000 columns).
      if (c.kernel == KF_ROWS_STREAM && narrow && c.stages <= 0) c.stages = 2;
    }
  }
  if (c.kernel == KF_ROWS_STREAM) {
    if (c.num_warps <= 0) c.num_warps = stream_default_warps(a.cols, elem);
    return c;
  }
  if (c.kernel == KF_ROWS_WARP) {
    c.num_warps = 1;  // warps per row
    return c;
  }
  const long long nvec = (a.cols * elem + 15) / 16;
  if (a.op == 0 && c.num_warps <= 0 && c.cluster <= 0 && nvec <= SOFTMAX_REGISTER_MAX_VECTORS) {
    // Softmax in registers: about eight 16-byte vectors per thread (a power
    // of two of warps, at most 16 vectors each), one CTA per row.
    long long w = 1;
    while (2 * w * 256 <= nvec) w *= 2;
    while (ceil_div(nvec, 32 * w) > 16) w *= 2;
    c.num_warps = static_cast<int>(w);
    c.cluster = 1;
  }
  if (c.cluster <= 0) {
    // One CTA holds up to 1024 threads x 4 vectors (64 KiB) of the row in registers.
    c.cluster = 1;
    if (nvec > 4096) {
      c.cluster = static_cast<int>((nvec + 4095) / 4096);
      if (c.cluster > 8) c.cluster = 8;
      // The next power of two keeps the cluster shape portable.
      int p2 = 1;
      while (p2 < c.cluster) p2 <<= 1;
      c.cluster = p2;
    }
  }
  if (c.num_warps <= 0) {
    const long long per_cta = (nvec + c.cluster - 1) / c.cluster;
    // About four 16-byte vectors per thread; a CTA holds at most 4096 vectors
    // whatever the split (1024 x 4, 512 x 8, 256 x 16), so wider rows need a
    // bigger cluster and fail the launch with "register pressure" beyond 8.
    long long threads = (per_cta + 3) / 4;
    if (threads > 1024) threads = 1024;
    long long warps = (threads + 31) / 32;
    if (warps < 1) warps = 1;
    if (warps > 32) warps = 32;
    c.num_warps = static_cast<int>(warps);
  }
  if (c.rows_per_cta <= 0) c.rows_per_cta = 1;
  return c;
}

int launch_rows(const RowsArgs& a, const kf_rows_config& cfg, const DeviceInfo& dev,
                cudaStream_t stream) {
  if (cfg.kernel == KF_ROWS_STREAM) return launch_rows_stream(a, cfg, dev, stream);
  if (cfg.kernel == KF_ROWS_WARP) return launch_rows_warp(a, dev, stream);
  if (cfg.kernel != KF_ROWS_REGISTER)
    return set_error(KF_ERR_INVALID_CONFIG, "kernel must be KF_ROWS_AUTO, _REGISTER, _STREAM or _WARP");
  if (cfg.num_warps < 1 || cfg.num_warps > 32)
    return set_error(KF_ERR_INVALID_CONFIG, "num_warps must be in [1, 32]");
  if (cfg.cluster < 1 || cfg.cluster > 8 || (cfg.cluster & (cfg.cluster - 1)) != 0)
    return set_error(KF_ERR_INVALID_CONFIG, "cluster must be 1, 2, 4 or 8");
  if (cfg.rows_per_cta < 1)
    return set_error(KF_ERR_INVALID_CONFIG, "rows_per_cta must be positive");
  if (a.cols > INT32_MAX) return set_error(KF_ERR_UNSUPPORTED, "row too wide");
  if (a.rows == 0 || a.cols == 0) return KF_OK;
  const long long clusters = (a.rows + cfg.rows_per_cta - 1) / cfg.rows_per_cta;
  if (clusters * cfg.cluster > INT32_MAX)
    return set_error(KF_ERR_UNSUPPORTED, "too many rows for one launch");
  if (a.op == OP_SOFTMAX) {
    switch (a.dtype) {
      case KF_FP16: return launch_typed<__half, OP_SOFTMAX>(a, cfg, stream);
      case KF_BF16: return launch_typed<__nv_bfloat16, OP_SOFTMAX>(a, cfg, stream);
      case KF_FP32: return launch_typed<float, OP_SOFTMAX>(a, cfg, stream);
    }
  } else {
    switch (a.dtype) {
      case KF_FP16: return launch_typed<__half, OP_RMSNORM>(a, cfg, stream);
      case KF_BF16: return launch_typed<__nv_bfloat16, OP_RMSNORM>(a, cfg, stream);
      case KF_FP32: return launch_typed<float, OP_RMSNORM>(a, cfg, stream);
    }
  }
  return set_error(KF_ERR_INVALID_ARGUMENT, "unknown dtype code");
}

}  // namespace kf
