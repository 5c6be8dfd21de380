// Row softmax and RMSNorm for narrow rows (up to 4 KB; the library's default
// up to 2 KB for softmax, 4 KB for RMSNorm), one warp per row.
//
// At 1000 fp16 columns a row is 2 KB: 125 vectors of 16 bytes, four per lane.
// The streaming kernel spends most of its issue slots on per-row machinery
// there -- a bulk copy and its mbarrier per row, the copy from shared memory
// to registers, one 512-thread CTA per SM held to it by registers (ncu: 67 %
// issue-active, 515 warp instructions per row, 16 warps per SM). This kernel
// has none of it: persistent CTAs of 8 warps, each warp owns rows w, w + W,
// w + 2W, ... (W = warps in the grid), and the lanes load the next row's
// vectors into registers (16-byte streaming loads) while they reduce and write
// the current one. No shared memory, no barriers: a row's statistic is a warp
// reduction. For RMSNorm each lane keeps its gamma vectors in registers for
// every row it handles.
//
// Rows must start on the 16-byte grid (input and output) and hold whole
// vectors; the library routes other layouts to the streaming or register
// kernels. Arithmetic as in rows_math.cuh: fp32 statistics, one ex2 per
// element, mixed-precision FMA for RMSNorm, one rounding of the output.
#include "kf_common.cuh"
#include "kf_internal.h"
#include "rows_math.cuh"

namespace kf {
namespace {

constexpr int WARP_ROW_WARPS = 8;

struct WarpRowsParams {
  const void* x;
  long long sx;
  const void* gamma;
  void* y;
  long long sy;
  long long rows;
  int nvec;  // 16-byte vectors per row
  float eps;
  float inv_cols;
};

template <typename T, int NV>
__device__ __forceinline__ void load_row(const WarpRowsParams& p, long long row, int lane, uint4 (&v)[NV]) {
  const uint4* xr = reinterpret_cast<const uint4*>(static_cast<const T*>(p.x) + row * p.sx);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = lane + 32 * j;
    v[j] = (row < p.rows && i < p.nvec) ? __ldcs(xr + i) : make_uint4(0u, 0u, 0u, 0u);
  }
}

template <typename T, int NV, int OP>
__global__ void __launch_bounds__(WARP_ROW_WARPS * 32) rows_warp_kernel(const WarpRowsParams p) {
  constexpr int VE = RowVec<T>::VE;
  const int lane = threadIdx.x & 31;
  const long long W = static_cast<long long>(gridDim.x) * WARP_ROW_WARPS;
  long long row = static_cast<long long>(blockIdx.x) * WARP_ROW_WARPS + (threadIdx.x >> 5);

  uint4 g[OP == 1 ? NV : 1];
  if constexpr (OP == 1) {
    const uint4* gv = reinterpret_cast<const uint4*>(p.gamma);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int i = lane + 32 * j;
      g[j] = i < p.nvec ? __ldg(gv + i) : make_uint4(0u, 0u, 0u, 0u);
    }
  }

  uint4 cur[NV], nxt[NV];
  load_row<T, NV>(p, row, lane, cur);
  for (; row < p.rows; row += W) {
    load_row<T, NV>(p, row + W, lane, nxt);  // the next row's loads go out first
    uint4* yr = reinterpret_cast<uint4*>(static_cast<T*>(p.y) + row * p.sy);
    if constexpr (OP == 0) {
      // softmax: (max, sum of exp) per lane, then over the warp
      uint4 mv = RowVec<T>::lowest();
#pragma unroll
      for (int j = 0; j < NV; ++j)
        if (lane + 32 * j < p.nvec) mv = vmax<T>(mv, cur[j]);
      const float m = hmax<T>(mv);
      // A lane whose elements are all -inf (or padding) has m = -inf: its
      // exponentials are 0, not exp(-inf + inf).
      const float mb = m == -INFINITY ? 0.0f : m * kRowLog2e;
      float ev[NV * VE];
      float s = 0.0f;
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        float f[VE];
        to_floats<T>(cur[j], f);
        const bool on = lane + 32 * j < p.nvec;
#pragma unroll
        for (int k = 0; k < VE; ++k) {
          ev[j * VE + k] = on ? ex2_ftz(fmaf(f[k], kRowLog2e, -mb)) : 0.0f;
          s += ev[j * VE + k];
        }
      }
      const float2 tot = warp_max_sum(m, s);  // a lane without elements has m = -inf and s = 0
      const float factor = m == -INFINITY ? 0.0f : ex2_ftz((m - tot.x) * kRowLog2e) * __frcp_rn(tot.y);
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        if (lane + 32 * j < p.nvec) {
          float o[VE];
#pragma unroll
          for (int k = 0; k < VE; ++k) o[k] = ev[j * VE + k] * factor;
          __stcs(yr + lane + 32 * j, from_floats<T>(o));
        }
      }
    } else {
      // RMSNorm: sum of squares without conversions (mixed-precision FMA)
      float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int j = 0; j < NV; ++j) acc = sumsq_vec<T>(cur[j], acc);  // padding vectors are zero
      const float scale = rsqrtf(warp_sum(acc.x + acc.y) * p.inv_cols + p.eps);
#pragma unroll
      for (int j = 0; j < NV; ++j)
        if (lane + 32 * j < p.nvec) __stcs(yr + lane + 32 * j, scale_gamma_vec<T>(cur[j], g[j], scale));
    }
#pragma unroll
    for (int j = 0; j < NV; ++j) cur[j] = nxt[j];
  }
}

template <typename T, int OP>
int launch_nv(const WarpRowsParams& p, const DeviceInfo& dev, cudaStream_t stream) {
  const int nv = (p.nvec + 31) / 32;
  void* fn = nv <= 1   ? reinterpret_cast<void*>(&rows_warp_kernel<T, 1, OP>)
             : nv <= 2 ? reinterpret_cast<void*>(&rows_warp_kernel<T, 2, OP>)
             : nv <= 4 ? reinterpret_cast<void*>(&rows_warp_kernel<T, 4, OP>)
                       : reinterpret_cast<void*>(&rows_warp_kernel<T, 8, OP>);
  static thread_local std::pair<void*, int> cached{nullptr, 0};
  int per_sm = 0;
  if (cached.first == fn) {
    per_sm = cached.second;
  } else {
    const cudaError_t err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, WARP_ROW_WARPS * 32, 0);
    if (err != cudaSuccess) return cuda_error(err, "cudaOccupancyMaxActiveBlocksPerMultiprocessor(rows_warp)");
    cached = {fn, per_sm};
  }
  if (per_sm < 1) per_sm = 1;
  long long blocks = (p.rows + WARP_ROW_WARPS - 1) / WARP_ROW_WARPS;
  const long long resident = static_cast<long long>(per_sm) * dev.sm_count;
  if (blocks > resident) blocks = resident;
  void* args[] = {const_cast<WarpRowsParams*>(&p)};
  const cudaError_t err =
      cudaLaunchKernel(fn, dim3(static_cast<unsigned>(blocks)), dim3(WARP_ROW_WARPS * 32), args, 0, stream);
  if (err != cudaSuccess) return cuda_error(err, "launch(rows_warp_kernel)");
  return KF_OK;
}

}  // namespace

bool rows_warp_supported(const RowsArgs& a, std::string* why) {
  const int elem = a.dtype == KF_FP32 ? 4 : 2;
  auto no = [&](const char* reason) {
    if (why) *why = reason;
    return false;
  };
  if ((a.cols * elem) % 16 != 0) return no("the warp-per-row kernel needs rows of whole 16-byte vectors");
  if ((a.cols * elem) / 16 > ROWS_WARP_EXPLICIT_MAX_VECTORS)
    return no("the warp-per-row kernel takes rows up to 4 KB");
  if ((reinterpret_cast<uintptr_t>(a.x) & 15u) != 0 || (reinterpret_cast<uintptr_t>(a.y) & 15u) != 0 ||
      (a.sx * elem) % 16 != 0 || (a.sy * elem) % 16 != 0)
    return no("the warp-per-row kernel needs rows that start on the 16-byte grid");
  if (a.op == 1 && (reinterpret_cast<uintptr_t>(a.gamma) & 15u) != 0)
    return no("the warp-per-row kernel needs a 16-byte-aligned gamma");
  return true;
}

int launch_rows_warp(const RowsArgs& a, const DeviceInfo& dev, cudaStream_t stream) {
  std::string why;
  if (!rows_warp_supported(a, &why)) return set_error(KF_ERR_UNALIGNED, why);
  if (a.rows == 0 || a.cols == 0) return KF_OK;
  WarpRowsParams p{};
  p.x = a.x;
  p.sx = a.sx;
  p.gamma = a.gamma;
  p.y = a.y;
  p.sy = a.sy;
  p.rows = a.rows;
  p.nvec = static_cast<int>(a.cols * (a.dtype == KF_FP32 ? 4 : 2) / 16);
  p.eps = a.eps;
  p.inv_cols = 1.0f / static_cast<float>(a.cols);
  if (a.op == 0) {
    switch (a.dtype) {
      case KF_FP16: return launch_nv<__half, 0>(p, dev, stream);
      case KF_BF16: return launch_nv<__nv_bfloat16, 0>(p, dev, stream);
      default: return launch_nv<float, 0>(p, dev, stream);
    }
  }
  switch (a.dtype) {
    case KF_FP16: return launch_nv<__half, 1>(p, dev, stream);
    case KF_BF16: return launch_nv<__nv_bfloat16, 1>(p, dev, stream);
    default: return launch_nv<float, 1>(p, dev, stream);
  }
}

}  // namespace kf
