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
// inside the row. Softmax reduces (max, sum of exp) pairs in one pass with the
// online rescaling rule sum = sum_a * exp(max_a - max) + sum_b * exp(max_b - max).
//
// Reference semantics: kernelforge/kernels/softmax.py:31-58 (max-shifted exp,
// fp32 math, output rounded once) and kernelforge/kernels/rmsnorm.py:41-72,
// 130-143 (fp32 sum of squares, x * rsqrt(mean + eps) * gamma, one rounding).
// The reference kernels cap rows at 16384 columns (search.py:459); these do not.
#include <cooperative_groups.h>

#include "kf_common.cuh"
#include "kf_internal.h"

namespace cg = cooperative_groups;

namespace kf {
namespace {

constexpr int OP_SOFTMAX = 0;
constexpr int OP_RMSNORM = 1;
// log2(e): exp(x) = 2^(x log2 e), so exponentials go through CUDA's exp2f.
constexpr float kLog2e = 1.4426950408889634f;

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

struct MaxSum {
  float m, s;
};

__device__ __forceinline__ MaxSum combine(MaxSum a, MaxSum b) {
  const float m = fmaxf(a.m, b.m);
  // An empty partial has m = -inf and s = 0; the guards keep -inf - -inf out.
  const float sa = a.m == m ? a.s : a.s * expf(a.m - m);
  const float sb = b.m == m ? b.s : b.s * expf(b.m - m);
  return {m, sa + sb};
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
      const uintptr_t addr = reinterpret_cast<uintptr_t>(xr);
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

    // ---- per-thread partial statistic
    float2 part;
    float ev[OP == OP_SOFTMAX ? NV * VE : 1];  // softmax: exp(x - m_local) per element
    float eh = 0.0f, et = 0.0f, m_local = 0.0f;
    if constexpr (OP == OP_SOFTMAX) {
      float m = -INFINITY;
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        if (g + j * G < nvec) {
#pragma unroll
          for (int e = 0; e < VE; ++e) m = fmaxf(m, to_f32(raw[j].e[e]));
        }
      }
      if (has_head) m = fmaxf(m, xh);
      if (has_tail) m = fmaxf(m, xt);
      // One exponential per element, relative to this thread's own maximum;
      // the values stay in registers and are rescaled by exp(m - M) / S once
      // the row's maximum M and sum S are known.
      float s = 0.0f;
      if (m != -INFINITY) {
#pragma unroll
        for (int j = 0; j < NV; ++j) {
          if (g + j * G < nvec) {
#pragma unroll
            for (int e = 0; e < VE; ++e) {
              const float t = exp2f((to_f32(raw[j].e[e]) - m) * kLog2e);
              ev[j * VE + e] = t;
              s += t;
            }
          }
        }
        if (has_head) {
          eh = exp2f((xh - m) * kLog2e);
          s += eh;
        }
        if (has_tail) {
          et = exp2f((xt - m) * kLog2e);
          s += et;
        }
      }
      m_local = m;
      part = make_float2(m, s);
    } else {
      float ss = 0.0f;
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        if (g + j * G < nvec) {
#pragma unroll
          for (int e = 0; e < VE; ++e) {
            const float f = to_f32(raw[j].e[e]);
            ss = fmaf(f, f, ss);
          }
        }
      }
      if (has_head) ss = fmaf(xh, xh, ss);
      if (has_tail) ss = fmaf(xt, xt, ss);
      part = make_float2(ss, 0.0f);
    }

    // ---- reduce: warp -> CTA -> cluster
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float a = __shfl_xor_sync(0xffffffffu, part.x, off);
      const float b = __shfl_xor_sync(0xffffffffu, part.y, off);
      if constexpr (OP == OP_SOFTMAX) {
        const MaxSum r = combine({part.x, part.y}, {a, b});
        part = make_float2(r.m, r.s);
      } else {
        part.x += a;
      }
    }
    if (lane == 0) warp_part[par][warp] = part;
    __syncthreads();
    float2 tot = warp_part[par][0];
    for (int w = 1; w < nwarps; ++w) {
      const float2 o = warp_part[par][w];
      if constexpr (OP == OP_SOFTMAX) {
        const MaxSum r = combine({tot.x, tot.y}, {o.x, o.y});
        tot = make_float2(r.m, r.s);
      } else {
        tot.x += o.x;
      }
    }
    if (csize > 1) {
      if (tid == 0) cta_part[par] = tot;
      cluster.sync();
      float2 all = *cluster.map_shared_rank(&cta_part[par], 0);
      for (unsigned r = 1; r < csize; ++r) {
        const float2 o = *cluster.map_shared_rank(&cta_part[par], r);
        if constexpr (OP == OP_SOFTMAX) {
          const MaxSum c = combine({all.x, all.y}, {o.x, o.y});
          all = make_float2(c.m, c.s);
        } else {
          all.x += o.x;
        }
      }
      tot = all;
    }

    // ---- normalise and store
    V* yv = reinterpret_cast<V*>(yr + head);
    if constexpr (OP == OP_SOFTMAX) {
      // exp(x - M) / S = exp(x - m_local) * (exp(m_local - M) / S)
      const float factor =
          m_local == -INFINITY ? 0.0f : exp2f((m_local - tot.x) * kLog2e) / tot.y;
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int v = g + j * G;
        if (v < nvec) {
          V o;
#pragma unroll
          for (int e = 0; e < VE; ++e) o.e[e] = from_f32<T>(ev[j * VE + e] * factor);
          store_stream(yv + v, o);
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
          V gv;
          if (gamma_vec) {
            gv = load_cached(reinterpret_cast<const V*>(gb) + v);
          } else {
#pragma unroll
            for (int e = 0; e < VE; ++e) gv.e[e] = gb[v * VE + e];
          }
          V o;
#pragma unroll
          for (int e = 0; e < VE; ++e)
            o.e[e] = from_f32<T>(to_f32(raw[j].e[e]) * scale * to_f32(gv.e[e]));
          store_stream(yv + v, o);
        }
      }
      if (has_head) yr[g] = from_f32<T>(xh * scale * to_f32(gamma[g]));
      if (has_tail) yr[tail_idx] = from_f32<T>(xt * scale * to_f32(gamma[tail_idx]));
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

kf_rows_config resolve_rows_config(const RowsArgs& a, const kf_rows_config* user) {
  kf_rows_config c{};
  if (user) c = *user;
  const int elem = a.dtype == KF_FP32 ? 4 : 2;
  const long long nvec = (a.cols * elem + 15) / 16;
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
  (void)dev;
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
