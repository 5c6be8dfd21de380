// extern "C" entry points of libkernelo_b200: argument checks, config
// resolution, dispatch to the tcgen05 / SIMT / row kernels, per-device caches
// and the device status word that bounded waits report timeouts into.
#include <array>
#include <mutex>
#include <string>

#include "kf_common.cuh"
#include "kf_internal.h"

// One status word per device context. Kernels whose bounded waits give up
// write KF_ERR_TIMEOUT | (site << 8) here; kf_device_status() reads and clears it.
__device__ int kf_status_word;

namespace kf {

namespace {
thread_local std::string g_last_error;
std::mutex g_dev_mutex;
std::array<DeviceInfo, 64> g_devices;
std::array<bool, 64> g_device_ready{};

__global__ void selftest_wait_kernel(int* status, unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    mbar_init_fence();
  }
  __syncthreads();
  // Nothing ever arrives on `bar`: the wait must give up on its own.
  if (threadIdx.x == 0) mbar_wait(smem_u32(&bar), 0, nullptr, status, SITE_SELFTEST, limit_ns);
}

bool valid_dtype(int d) { return d == KF_FP16 || d == KF_BF16 || d == KF_FP32; }

kf_gemm_config zero_config() {
  kf_gemm_config c{};
  return c;
}
}  // namespace

int set_error(int code, const std::string& message) {
  g_last_error = message;
  return code;
}

int cuda_error(cudaError_t err, const char* where) {
  const std::string msg = std::string(where) + ": " + cudaGetErrorString(err);
  switch (err) {
    case cudaErrorLaunchOutOfResources:
    case cudaErrorInvalidConfiguration:
    case cudaErrorInvalidClusterSize:
      return set_error(KF_ERR_INVALID_CONFIG, msg);
    case cudaErrorNoDevice:
    case cudaErrorInsufficientDriver:
    case cudaErrorNoKernelImageForDevice:
      return set_error(KF_ERR_NO_DEVICE, msg);
    default:
      return set_error(KF_ERR_LAUNCH, msg);
  }
}

int current_device(int* device) {
  cudaError_t err = cudaGetDevice(device);
  if (err != cudaSuccess) return cuda_error(err, "cudaGetDevice");
  return KF_OK;
}

int device_info(int device, DeviceInfo** out) {
  if (device < 0 || device >= static_cast<int>(g_devices.size()))
    return set_error(KF_ERR_INVALID_ARGUMENT, "device index out of range");
  std::lock_guard<std::mutex> lock(g_dev_mutex);
  if (!g_device_ready[device]) {
    int prev = 0;
    cudaError_t err = cudaGetDevice(&prev);
    if (err != cudaSuccess) return cuda_error(err, "cudaGetDevice");
    if (prev != device) {
      err = cudaSetDevice(device);
      if (err != cudaSuccess) return cuda_error(err, "cudaSetDevice");
    }
    DeviceInfo info;
    cudaDeviceProp prop;
    err = cudaGetDeviceProperties(&prop, device);
    if (err == cudaSuccess) {
      info.sm_count = prop.multiProcessorCount;
      info.max_smem_optin = static_cast<int>(prop.sharedMemPerBlockOptin);
      info.major = prop.major;
      info.minor = prop.minor;
      void* addr = nullptr;
      err = cudaGetSymbolAddress(&addr, kf_status_word);
      info.status = static_cast<int*>(addr);
    }
    if (prev != device) cudaSetDevice(prev);
    if (err != cudaSuccess) return cuda_error(err, "device_info");
    if (info.major != 10)
      return set_error(KF_ERR_NO_DEVICE, "libkernelo_b200 is built for sm_100a; device " +
                                             std::to_string(device) + " is sm_" +
                                             std::to_string(info.major) +
                                             std::to_string(info.minor));
    g_devices[device] = info;
    g_device_ready[device] = true;
  }
  *out = &g_devices[device];
  return KF_OK;
}

kf_gemm_config resolve_gemm_config(const GemmArgs& g, const kf_gemm_config* user, int sm_count) {
  kf_gemm_config c = user ? *user : zero_config();
  const bool tc_ok = tcgen05_operands_ok(g, nullptr);
  if (c.kernel == KF_GEMM_AUTO) c.kernel = tc_ok ? KF_GEMM_TCGEN05 : KF_GEMM_SIMT;
  if (c.kernel == KF_GEMM_SIMT) {
    if (c.block_m == 0 && c.block_n == 0 && c.block_k == 0) {
      const bool small = g.M * g.N < 128LL * 128 * sm_count;
      c.block_m = small ? 64 : 128;
      c.block_n = small ? 64 : 128;
      c.block_k = small ? 16 : 8;
    }
    return c;
  }
  // tcgen05 defaults.
  if (c.swap_ab == 0) c.swap_ab = (g.M <= 64 && g.N > g.M) ? 1 : 2;
  const bool swap = c.swap_ab == 1;
  const int64_t m = swap ? g.N : g.M;
  const int64_t n = swap ? g.M : g.N;
  // B' is MN-major when its N' index has unit stride.
  const int64_t sb_c = swap ? g.sa_m : g.sb_n;
  const int64_t sb_k = swap ? g.sa_k : g.sb_k;
  const bool b_mn = !(sb_k == 1) && sb_c == 1;
  if (c.block_m == 0) {
    // An SM pair (256-row tiles, pair MMA) whenever 256 x 256 tiles still give
    // every pair work; it halves each SM's shared-memory traffic for B.
    const int64_t pair_tiles = ((m + 255) / 256) * ((n + 255) / 256);
    c.block_m = (m >= 256 && n >= 128 && c.stream_k != 1 && pair_tiles >= sm_count / 2) ? 256 : 128;
  }
  const int cg = c.block_m == 256 ? 2 : 1;
  if (c.block_n == 0) {
    const int quantum = (b_mn ? 64 : 16) * cg;
    // TF32 tiles sum their accumulator chunks in registers: at most 128 wide.
    const int64_t widest = g.dtype == KF_FP32 ? 128 : 256;
    int64_t bn = n <= widest ? ((n + quantum - 1) / quantum) * quantum : widest;
    if (bn < quantum) bn = quantum;
    if (bn > 256) bn = 256;
    c.block_n = static_cast<int32_t>(bn);
  }
  // Pair tiles: two 128-byte atoms of K per k-block halve the barrier round
  // trips per FLOP (measured faster than one atom at equal bytes in flight).
  // An atom is 64 16-bit or 32 fp32 (TF32) elements.
  const int elem = g.dtype == KF_FP32 ? 4 : 2;
  const int atom = 128 / elem;
  // bytes per (row, k) in a ring stage and in an A panel: TF32 stages carry
  // both split parts of each element
  const int stage_elem = g.dtype == KF_FP32 ? 2 * elem : elem;
  // (TF32 pairs too: two 96 KB stages of 64-deep k-blocks beat four of 32,
  // 466 against 501 us at 2048 x 4096 x 4096 and 921 against 982 at 4099^3)
  if (c.block_k == 0) c.block_k = (cg == 2 && g.K >= 512) ? 2 * atom : atom;
  if (c.stages == 0) {
    const int64_t per_stage = static_cast<int64_t>(128 + c.block_n / cg) * c.block_k * stage_elem;
    // (the all-gather epilogue's output stage comes out of the same 227 KiB)
    int64_t s = (232448 - 1024 - 256 - (g.n_peers > 0 ? GEMM_PEER_STAGE_SMEM : 0)) / per_stage;
    if (s > 12) s = 12;
    if (s < 2) s = 2;
    c.stages = static_cast<int32_t>(s);
  }
  if (c.group_m == 0) {
    // Grouped raster width: as many M tiles as keep their A panels (the whole
    // K extent) within ~48 MB of L2, so that each group streams B once and A
    // stays resident across waves (measured on B200 at 4096x11008x4096: 16
    // groups-of-one-column read B once, 8 read it twice and ran 3 % slower).
    const int64_t tile_rows = 128LL * cg;
    const int64_t panel = tile_rows * g.K * stage_elem;
    int64_t gm = panel > 0 ? (48LL << 20) / panel : 8;
    const int64_t tiles_m = (m + tile_rows - 1) / tile_rows;
    if (gm > tiles_m) gm = tiles_m;
    if (gm < 1) gm = 1;
    c.group_m = static_cast<int32_t>(gm);
  }
  if (c.stream_k == 0) {
    // Fewer one-SM tiles than SMs and a long K (decode shapes, the swapped
    // GEMV): all stream-K. Fewer tiles than SMs and a short K (or too few
    // k-blocks in all for 8 per SM, where stream-K's fix-up would gather a
    // dozen partials per tile): narrower
    // tiles, whole (at 1021 x 2053 x 509 and 257^3 whole 64-column tiles
    // measured 1.6-2x faster than stream-K, whose fix-up a few k-blocks
    // cannot pay for). Otherwise the split tail: whole tiles for the full
    // waves, the last partial wave as half-width tiles (at 4096x11008x4096:
    // 688 pair tiles on 74 pairs leave 22 for the last wave; a stream-K tail
    // measured slower there, its fix-up epilogues all falling at the end).
    const int64_t tiles_m = (m + 128LL * cg - 1) / (128LL * cg);
    int64_t tiles = tiles_m * ((n + c.block_n - 1) / c.block_n);
    const int64_t kb = (g.K + c.block_k - 1) / c.block_k;
    if (kb < 4) {
      c.stream_k = 2;
    } else if (cg == 1 && tiles < sm_count && (kb < 16 || tiles * kb < 8LL * sm_count)) {
      const int quantum = b_mn ? 64 : 16;
      const bool user_bn = user != nullptr && user->block_n != 0;
      for (const int bn : {128, 64}) {
        if (user_bn || tiles >= sm_count || bn >= c.block_n || bn % quantum != 0) continue;
        c.block_n = bn;
        tiles = tiles_m * ((n + bn - 1) / bn);
      }
      c.stream_k = 2;
    } else {
      c.stream_k = (cg == 1 && tiles < sm_count) ? 1 : 3;
    }
  }
  if (cg == 2 && c.cluster_m == 0) c.cluster_m = 2;
  return c;
}

}  // namespace kf

using namespace kf;

namespace {

// ---- the tcgen05 path's workspace plan ------------------------------------
// fp16/bf16 operands a TMA tensor map cannot describe (a row pitch or base off
// the 16-byte grid: K = 4099, N = 2053, a view starting at an odd column; or
// K < 8) are copied into the caller's workspace as pitched matrices and the
// tcgen05 kernel runs on the copies (pack.cu). An output whose rows are off
// the 16-byte grid is written to a pitched copy with vector stores and moved
// to C by one copy kernel. Workspace layout:
//   [stream-K region, at least its 64 KiB of counters | packed A | packed B | staged C]
// so the counters a later stream-K call relies on are never overwritten.
struct TcPlan {
  bool pack_a = false, pack_b = false, stage_c = false;
  bool split = false;  // fp32: both operands split into TF32 parts (3xTF32)
  PackedOperand a, b, c;
  SplitOperand sa, sb;
  GemmArgs view;  // the problem as the kernel sees it (packed operands' strides)
  kf_gemm_config cfg{};
  int64_t sk = 0;  // stream-K bytes
  int64_t offset() const {
    const int64_t r = (sk + 255) / 256 * 256;
    return r > SK_COUNTER_BYTES ? r : SK_COUNTER_BYTES;
  }
  int64_t staging_bytes() const {
    if (split) return sa.bytes + sb.bytes;
    return (pack_a ? a.bytes : 0) + (pack_b ? b.bytes : 0) + (stage_c ? c.bytes : 0);
  }
  int64_t need() const { return staging_bytes() > 0 ? offset() + staging_bytes() : sk; }
};

// Packing pays where the GEMM is compute-bound: both M and N above 64 (a
// skinny problem keeps the CUDA-core kernel, which reads its operands in
// place), or when tcgen05 is asked for explicitly.
bool packing_applies(const GemmArgs& g, const kf_gemm_config* user) {
  if (g.dtype == KF_FP32 || g.n_peers > 0 || g.K == 0) return false;
  const int kernel = user ? user->kernel : KF_GEMM_AUTO;
  if (kernel != KF_GEMM_AUTO && kernel != KF_GEMM_TCGEN05) return false;
  if (tcgen05_operands_ok(g, nullptr)) return false;
  return kernel == KF_GEMM_TCGEN05 || (g.M > 64 && g.N > 64);
}

// fp32 on tensor cores (3xTF32, tf32_split.cu) where the GEMM is
// compute-bound: both M and N above 64 and at least 2^27 multiply-adds, or
// tcgen05 asked for explicitly. Smaller fp32 problems keep the CUDA-core
// kernel (IEEE FMA in place, one launch instead of three: at 257^3 it measured
// 28.8 us against 31.8 for split + TF32 GEMM).
constexpr int64_t TF32_MIN_MACS = int64_t{1} << 27;
bool tf32_applies(const GemmArgs& g, const kf_gemm_config* user) {
  if (g.dtype != KF_FP32 || g.n_peers > 0 || g.K == 0) return false;
  const int kernel = user ? user->kernel : KF_GEMM_AUTO;
  if (kernel == KF_GEMM_TCGEN05) return true;
  return kernel == KF_GEMM_AUTO && g.M > 64 && g.N > 64 && g.M * g.N * g.K >= TF32_MIN_MACS;
}

// Whether the epilogue's 16-byte stores cannot reach C: its rows are off the
// 16-byte grid (an odd N, a view starting at an odd column). Swapped (skinny)
// tiles write C's columns and keep their element stores.
bool output_needs_stage(const GemmArgs& v, const kf_gemm_config& cfg) {
  if (v.dtype == KF_FP32 || v.n_peers > 0 || cfg.swap_ab == 1 || v.M <= 64 || v.N < 16) return false;
  return !(v.sc_n == 1 && (v.sc_m * 2) % 16 == 0 && (reinterpret_cast<uintptr_t>(v.c) & 15u) == 0);
}

// The plan of a tcgen05 call with `have` bytes of workspace (-1: as much as it
// needs). Returns false when the call cannot take tcgen05 (operands to pack
// and too little workspace); an explicit tcgen05 request then fails.
bool plan_tc(const GemmArgs& g, const kf_gemm_config* user, const DeviceInfo& dev, int64_t have, TcPlan* out) {
  TcPlan& p = *out;
  p.view = g;
  const void* stand_in = reinterpret_cast<const void*>(static_cast<uintptr_t>(256));
  if (tf32_applies(g, user)) {
    // A'[M, 2Kp] and B'[N, 2Kp] ([small | big] rows), both K-major: the
    // kernel's K is Kp and each k-block loads both segments.
    p.split = true;
    p.sa = plan_tf32_split(g.a, g.sa_m, g.sa_k, g.M, g.K);
    p.sb = plan_tf32_split(g.b, g.sb_n, g.sb_k, g.N, g.K);
    p.view.a = stand_in;
    p.view.sa_m = p.sa.pitch;
    p.view.sa_k = 1;
    p.view.b = stand_in;
    p.view.sb_n = p.sb.pitch;
    p.view.sb_k = 1;
    p.view.K = p.sa.kp;
    p.view.tf32_split = true;
  } else if (packing_applies(g, user)) {
    // K below one 16-byte vector is padded with zeros to 8: then both operands
    // need the padded extent, so both are copied.
    const int64_t kp = g.K < 8 ? 8 : g.K;
    p.pack_a = kp != g.K || !tma_describable(g.a, g.sa_m, g.sa_k, g.M, g.K);
    p.pack_b = kp != g.K || !tma_describable(g.b, g.sb_n, g.sb_k, g.N, g.K);
    // Stand-in aligned pointers until the workspace is known: only strides and
    // sizes decide the config.
    if (p.pack_a) {
      p.a = plan_pack(g.a, g.sa_m, g.sa_k, g.M, g.K, kp);
      p.view.a = stand_in;
      p.view.sa_m = p.a.k_inner ? p.a.pitch : 1;
      p.view.sa_k = p.a.k_inner ? 1 : p.a.pitch;
    }
    if (p.pack_b) {
      p.b = plan_pack(g.b, g.sb_n, g.sb_k, g.N, g.K, kp);
      p.view.b = stand_in;
      p.view.sb_n = p.b.k_inner ? p.b.pitch : 1;
      p.view.sb_k = p.b.k_inner ? 1 : p.b.pitch;
    }
    p.view.K = kp;
  }
  p.cfg = resolve_gemm_config(p.view, user, dev.sm_count);
  if (p.cfg.kernel != KF_GEMM_TCGEN05) return false;
  p.stage_c = output_needs_stage(p.view, p.cfg);
  if (p.stage_c) p.c = plan_output_stage(g.c, g.sc_m, g.sc_n, g.M, g.N);
  p.sk = p.cfg.stream_k == 1 ? gemm_tcgen05_workspace_bytes(p.view, p.cfg, dev) : 0;
  if (have < 0) return true;
  const bool library_sk = user == nullptr || user->stream_k == 0;
  // What gives way when the workspace is short: the library's own stream-K
  // choice (whole tiles instead), then the output staging (element stores).
  if (p.need() > have && p.sk > 0 && library_sk) {
    p.cfg.stream_k = 2;
    p.sk = 0;
  }
  if (p.need() > have && p.stage_c) p.stage_c = false;
  return p.need() <= have;
}

int gemm_common(GemmArgs& g, const kf_gemm_config* user, void* stream) {
  if (!valid_dtype(g.dtype)) return set_error(KF_ERR_INVALID_ARGUMENT, "unknown dtype code");
  if (g.M < 0 || g.N < 0 || g.K < 0) return set_error(KF_ERR_INVALID_ARGUMENT, "negative size");
  if (g.M == 0 || g.N == 0) return KF_OK;
  if (g.c == nullptr || (g.K > 0 && (g.a == nullptr || g.b == nullptr)))
    return set_error(KF_ERR_INVALID_ARGUMENT, "null operand pointer");
  if (g.epilogue != KF_EPI_NONE && g.bias == nullptr)
    return set_error(KF_ERR_INVALID_ARGUMENT, "epilogue needs a bias pointer");
  if (g.epilogue < KF_EPI_NONE || g.epilogue > KF_EPI_BIAS_GELU_ERF)
    return set_error(KF_ERR_INVALID_ARGUMENT, "unknown epilogue code");
  // Up to 32 rows of x against a K-contiguous 16-bit B (an nn.Linear weight
  // [N, K] passed as its transpose): the 16-row tile kernel, epilogue and
  // peer stores included (the decode-shape fused linear and its all-gather).
  // It reads the weight at 0.8 of the copy bandwidth against ~0.55 for
  // 128-row TMA tiles.
  if (user != nullptr && user->kernel == KF_GEMM_TILE_STREAM) {
    if (g.n_peers != 0 || g.sync != nullptr)
      return set_error(KF_ERR_UNSUPPORTED, "streamed tile GEMV: no peer stores (use the tile kernel)");
    std::string why;
    if (!gemv_stream_supported(g.dtype, g.a, g.sa_m, g.sa_k, g.b, g.sb_n, g.sb_k, g.M, g.N, g.K, &why))
      return set_error(g.M > GEMV_STREAM_MAX_M ? KF_ERR_UNSUPPORTED : KF_ERR_UNALIGNED, "streamed tile GEMV: " + why);
    int device = 0;
    int rc = current_device(&device);
    if (rc != KF_OK) return rc;
    DeviceInfo* dev = nullptr;
    rc = device_info(device, &dev);
    if (rc != KF_OK) return rc;
    return launch_gemv_stream(g.dtype, g.a, g.sa_m, g.b, g.sb_n, g.c, g.sc_m, g.sc_n, g.M, g.N, g.K, *user, *dev,
                              static_cast<cudaStream_t>(stream), g.epilogue, g.bias);
  }
  // The library's decode-shape choice between the two 16-row tile kernels.
  if ((user == nullptr || user->kernel == KF_GEMM_AUTO) && g.n_peers == 0 && g.sync == nullptr &&
      g.M <= GEMV_STREAM_MAX_M &&
      gemv_stream_supported(g.dtype, g.a, g.sa_m, g.sa_k, g.b, g.sb_n, g.sb_k, g.M, g.N, g.K, nullptr)) {
    int device = 0;
    int rc = current_device(&device);
    if (rc != KF_OK) return rc;
    DeviceInfo* dev = nullptr;
    rc = device_info(device, &dev);
    if (rc != KF_OK) return rc;
    const int overlap = user != nullptr ? user->overlap : 0;
    if (gemv_stream_preferred(g.M, g.N, g.K, dev->sm_count, overlap != 0)) {
      kf_gemm_config chosen = zero_config();
      chosen.kernel = KF_GEMM_TILE_STREAM;
      chosen.overlap = overlap;
      return launch_gemv_stream(g.dtype, g.a, g.sa_m, g.b, g.sb_n, g.c, g.sc_m, g.sc_n, g.M, g.N, g.K, chosen,
                                *dev, static_cast<cudaStream_t>(stream), g.epilogue, g.bias);
    }
  }
  const bool tile_auto = (user == nullptr || user->kernel == KF_GEMM_AUTO) && g.M <= GEMV_MMA_MAX_M &&
                         gemv_mma_supported(g.dtype, g.a, g.sa_m, g.sa_k, g.b, g.sb_n, g.sb_k, g.M, g.N,
                                            g.K, nullptr);
  if (tile_auto || (user != nullptr && user->kernel == KF_GEMM_TILE_ROWS)) {
    std::string why;
    if (!gemv_mma_supported(g.dtype, g.a, g.sa_m, g.sa_k, g.b, g.sb_n, g.sb_k, g.M, g.N, g.K, &why))
      return set_error(KF_ERR_UNALIGNED, "tile GEMV: " + why);
    // The library's own choice ignores the other config fields (they describe
    // tcgen05 tiles when the kernel was left to the library).
    int* status = nullptr;
    if (g.sync != nullptr) {  // the barrier runs in the kernel's last CTA
      int device = 0;
      int rc = current_device(&device);
      if (rc != KF_OK) return rc;
      DeviceInfo* dev = nullptr;
      rc = device_info(device, &dev);
      if (rc != KF_OK) return rc;
      status = dev->status;
    }
    const int rc = launch_gemv_mma(g.dtype, g.a, g.sa_m, g.b, g.sb_n, g.c, g.sc_m, g.sc_n, g.M, g.N, g.K,
                                   tile_auto ? zero_config() : *user, static_cast<cudaStream_t>(stream),
                                   g.epilogue, g.bias, g.peers, g.n_peers, g.sync, status);
    if (rc == KF_OK && g.sync != nullptr) g.sync_done = true;
    return rc;
  }
  // Up to 8 rows of x against an N-contiguous B (the reference's row-major
  // (K, N) operand): lanes stream B's rows in 512-byte warp loads, K split
  // over CTAs.
  const bool cols_auto = (user == nullptr || user->kernel == KF_GEMM_AUTO) && g.n_peers == 0 &&
                         gemv_cols_supported(g.dtype, g.a, g.b, g.sb_k, g.sb_n, g.M, g.N, g.K, nullptr);
  if (cols_auto || (user != nullptr && user->kernel == KF_GEMM_COLUMNS)) {
    if (g.n_peers > 0) return set_error(KF_ERR_UNSUPPORTED, "the column GEMV has no all-gather epilogue");
    std::string why;
    if (!gemv_cols_supported(g.dtype, g.a, g.b, g.sb_k, g.sb_n, g.M, g.N, g.K, &why))
      return set_error(KF_ERR_UNALIGNED, why);
    int device = 0;
    int rc = current_device(&device);
    if (rc != KF_OK) return rc;
    DeviceInfo* dev = nullptr;
    rc = device_info(device, &dev);
    if (rc != KF_OK) return rc;
    return launch_gemv_cols(g.dtype, g.a, g.sa_m, g.sa_k, g.b, g.sb_k, g.c, g.sc_m, g.sc_n, g.M, g.N, g.K,
                            g.epilogue, g.bias, g.workspace, g.workspace_bytes, dev->sm_count,
                            static_cast<cudaStream_t>(stream));
  }
  if (g.n_peers > 0 && !tcgen05_operands_ok(g, nullptr))
    return set_error(KF_ERR_UNALIGNED,
                     "the all-gather epilogue needs TMA-describable operands (or the tile GEMV's, M <= 32)");
  int device = 0;
  int rc = current_device(&device);
  if (rc != KF_OK) return rc;
  DeviceInfo* dev = nullptr;
  rc = device_info(device, &dev);
  if (rc != KF_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t have = g.workspace != nullptr ? g.workspace_bytes : 0;
  TcPlan plan;
  if (plan_tc(g, user, *dev, have, &plan)) {
    GemmArgs& v = plan.view;
    char* dst = static_cast<char*>(g.workspace) + plan.offset();
    if (plan.split) {
      rc = launch_tf32_split(plan.sa, dst, s);
      if (rc != KF_OK) return rc;
      v.a = dst;
      dst += plan.sa.bytes;
      rc = launch_tf32_split(plan.sb, dst, s);
      if (rc != KF_OK) return rc;
      v.b = dst;
      dst += plan.sb.bytes;
    }
    if (plan.pack_a) {
      rc = launch_pack(plan.a, dst, s);
      if (rc != KF_OK) return rc;
      v.a = dst;
      dst += plan.a.bytes;
    }
    if (plan.pack_b) {
      rc = launch_pack(plan.b, dst, s);
      if (rc != KF_OK) return rc;
      v.b = dst;
      dst += plan.b.bytes;
    }
    if (plan.stage_c) {
      v.c = dst;
      v.sc_m = plan.c.pitch;
      v.sc_n = 1;
    }
    v.workspace = plan.sk > 0 ? g.workspace : nullptr;
    v.workspace_bytes = plan.sk;
    rc = launch_gemm_tcgen05(v, plan.cfg, *dev, s);
    if (rc != KF_OK || !plan.stage_c) return rc;
    return launch_unpack(plan.c, dst, s);
  }
  if (plan.pack_a || plan.pack_b || plan.split) {
    if (user != nullptr && user->kernel == KF_GEMM_TCGEN05)
      return set_error(KF_ERR_WORKSPACE,
                       std::string(plan.split ? "fp32 operands are split into TF32 parts first"
                                              : "operands TMA cannot describe are packed first") +
                           ": this call needs " + std::to_string(plan.need()) + " bytes of workspace, got " +
                           std::to_string(have));
    // no room to pack or split: the CUDA-core kernel reads the operands in place
  }
  // (an explicit stream-K request without enough workspace is refused by the launch)
  kf_gemm_config cfg = resolve_gemm_config(g, user, dev->sm_count);
  if (cfg.kernel == KF_GEMM_TCGEN05) return launch_gemm_tcgen05(g, cfg, *dev, s);
  if (cfg.kernel == KF_GEMM_SIMT) {
    if (g.n_peers > 0)
      return set_error(KF_ERR_UNSUPPORTED, "the all-gather epilogue is on the tcgen05 and tile GEMV paths only");
    return launch_gemm_simt(g, cfg, s);
  }
  return set_error(KF_ERR_INVALID_CONFIG, "unknown GEMM kernel code");
}

}  // namespace

extern "C" {

int32_t kf_abi_version(void) { return KF_ABI_VERSION; }

const char* kf_version(void) { return "kernelo_b200 0.1.0 (sm_100a)"; }

const char* kf_last_error(void) { return g_last_error.c_str(); }

int32_t kf_sm_count(int32_t device) {
  DeviceInfo* dev = nullptr;
  const int rc = device_info(device, &dev);
  if (rc != KF_OK) return -rc;
  return dev->sm_count;
}

int32_t kf_device_status(int32_t device, int32_t* out) {
  if (out == nullptr) return set_error(KF_ERR_INVALID_ARGUMENT, "null out pointer");
  DeviceInfo* dev = nullptr;
  int rc = device_info(device, &dev);
  if (rc != KF_OK) return rc;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(device);
  int value = 0;
  cudaError_t err = cudaDeviceSynchronize();
  if (err == cudaSuccess) err = cudaMemcpyFromSymbol(&value, kf_status_word, sizeof(int));
  const int zero = 0;
  if (err == cudaSuccess) err = cudaMemcpyToSymbol(kf_status_word, &zero, sizeof(int));
  cudaSetDevice(prev);
  if (err != cudaSuccess) return cuda_error(err, "kf_device_status");
  *out = value;
  return KF_OK;
}

int32_t kf_gemm(int32_t dtype, const void* a, int64_t sa_m, int64_t sa_k, const void* b,
                int64_t sb_k, int64_t sb_n, void* c, int64_t sc_m, int64_t sc_n, int64_t M,
                int64_t N, int64_t K, const kf_gemm_config* cfg, void* workspace,
                int64_t workspace_bytes, void* stream) {
  GemmArgs g;
  g.dtype = dtype;
  g.a = a;
  g.sa_m = sa_m;
  g.sa_k = sa_k;
  g.b = b;
  g.sb_k = sb_k;
  g.sb_n = sb_n;
  g.c = c;
  g.sc_m = sc_m;
  g.sc_n = sc_n;
  g.M = M;
  g.N = N;
  g.K = K;
  g.workspace = workspace;
  g.workspace_bytes = workspace_bytes;
  return gemm_common(g, cfg, stream);
}

int32_t kf_linear_bias_act(int32_t dtype, const void* x, int64_t sx_m, int64_t sx_k,
                           const void* w, int64_t sw_k, int64_t sw_n, const void* bias, void* y,
                           int64_t sy_m, int64_t sy_n, int64_t M, int64_t N, int64_t K,
                           int32_t epilogue, const kf_gemm_config* cfg, void* workspace,
                           int64_t workspace_bytes, void* stream) {
  GemmArgs g;
  g.dtype = dtype;
  g.a = x;
  g.sa_m = sx_m;
  g.sa_k = sx_k;
  g.b = w;
  g.sb_k = sw_k;
  g.sb_n = sw_n;
  g.c = y;
  g.sc_m = sy_m;
  g.sc_n = sy_n;
  g.M = M;
  g.N = N;
  g.K = K;
  g.bias = bias;
  g.epilogue = epilogue;
  g.workspace = workspace;
  g.workspace_bytes = workspace_bytes;
  return gemm_common(g, cfg, stream);
}

}  // extern "C"

static int allgather_impl(int32_t dtype, const void* x, int64_t sx_m, int64_t sx_k, const void* w, int64_t sw_k,
                          int64_t sw_n, const void* bias, void* y, int64_t sy_m, int64_t sy_n, int64_t M, int64_t N,
                          int64_t K, int32_t epilogue, void* const* y_peers, int32_t n_peers,
                          const kf_peer_sync* sync, const kf_gemm_config* cfg, void* workspace,
                          int64_t workspace_bytes, void* stream) {
  if (n_peers < 0 || n_peers > KF_MAX_PEERS)
    return set_error(KF_ERR_INVALID_ARGUMENT,
                     "n_peers must be in [0, " + std::to_string(KF_MAX_PEERS) + "]");
  if (n_peers > 0 && y_peers == nullptr) return set_error(KF_ERR_INVALID_ARGUMENT, "null y_peers");
  if (cfg != nullptr && cfg->kernel == KF_GEMM_SIMT && n_peers > 0)
    return set_error(KF_ERR_UNSUPPORTED, "the all-gather epilogue is on the tcgen05 and tile GEMV paths only");
  GemmArgs g;
  g.dtype = dtype;
  g.a = x;
  g.sa_m = sx_m;
  g.sa_k = sx_k;
  g.b = w;
  g.sb_k = sw_k;
  g.sb_n = sw_n;
  g.c = y;
  g.sc_m = sy_m;
  g.sc_n = sy_n;
  g.M = M;
  g.N = N;
  g.K = K;
  g.bias = bias;
  g.epilogue = epilogue;
  g.workspace = workspace;
  g.workspace_bytes = workspace_bytes;
  g.n_peers = n_peers;
  for (int i = 0; i < n_peers; ++i) {
    if (y_peers[i] == nullptr) return set_error(KF_ERR_INVALID_ARGUMENT, "null peer output pointer");
    g.peers[i] = y_peers[i];
  }
  g.sync = sync;
  int rc = gemm_common(g, cfg, stream);
  if (rc != KF_OK || sync == nullptr || g.sync_done) return rc;
  // the tcgen05 path (or an empty output): the barrier kernel follows
  int device = 0;
  rc = current_device(&device);
  if (rc != KF_OK) return rc;
  DeviceInfo* dev = nullptr;
  rc = device_info(device, &dev);
  if (rc != KF_OK) return rc;
  return launch_peer_barrier(sync->local_signals, sync->peer_signals, sync->rank, sync->world, 0, sync->timeout_us,
                             *dev, static_cast<cudaStream_t>(stream), sync->epoch_counter);
}


extern "C" {

int32_t kf_linear_bias_act_allgather(int32_t dtype, const void* x, int64_t sx_m, int64_t sx_k,
                                     const void* w, int64_t sw_k, int64_t sw_n, const void* bias,
                                     void* y, int64_t sy_m, int64_t sy_n, int64_t M, int64_t N,
                                     int64_t K, int32_t epilogue, void* const* y_peers,
                                     int32_t n_peers, const kf_gemm_config* cfg, void* workspace,
                                     int64_t workspace_bytes, void* stream) {
  return allgather_impl(dtype, x, sx_m, sx_k, w, sw_k, sw_n, bias, y, sy_m, sy_n, M, N, K, epilogue, y_peers, n_peers,
                        nullptr, cfg, workspace, workspace_bytes, stream);
}

int32_t kf_linear_bias_act_allgather_sync(int32_t dtype, const void* x, int64_t sx_m, int64_t sx_k,
                                          const void* w, int64_t sw_k, int64_t sw_n, const void* bias, void* y,
                                          int64_t sy_m, int64_t sy_n, int64_t M, int64_t N, int64_t K,
                                          int32_t epilogue, void* const* y_peers, int32_t n_peers,
                                          const kf_peer_sync* sync, const kf_gemm_config* cfg, void* workspace,
                                          int64_t workspace_bytes, void* stream) {
  if (sync == nullptr) return set_error(KF_ERR_INVALID_ARGUMENT, "null peer sync");
  if (sync->epoch_counter == nullptr) return set_error(KF_ERR_INVALID_ARGUMENT, "null epoch counter");
  return allgather_impl(dtype, x, sx_m, sx_k, w, sw_k, sw_n, bias, y, sy_m, sy_n, M, N, K, epilogue, y_peers, n_peers,
                        sync, cfg, workspace, workspace_bytes, stream);
}

int32_t kf_peer_barrier(uint32_t* local_signals, uint32_t* const* peer_signals, int32_t rank,
                        int32_t world, uint32_t epoch, int32_t timeout_us, void* stream) {
  int device = 0;
  int rc = current_device(&device);
  if (rc != KF_OK) return rc;
  DeviceInfo* dev = nullptr;
  rc = device_info(device, &dev);
  if (rc != KF_OK) return rc;
  return launch_peer_barrier(local_signals, peer_signals, rank, world, epoch, timeout_us, *dev,
                             static_cast<cudaStream_t>(stream));
}

int32_t kf_peer_barrier_counted(uint32_t* local_signals, uint32_t* const* peer_signals, int32_t rank,
                                int32_t world, uint32_t* epoch_counter, int32_t timeout_us, void* stream) {
  if (epoch_counter == nullptr) return set_error(KF_ERR_INVALID_ARGUMENT, "null epoch counter");
  int device = 0;
  int rc = current_device(&device);
  if (rc != KF_OK) return rc;
  DeviceInfo* dev = nullptr;
  rc = device_info(device, &dev);
  if (rc != KF_OK) return rc;
  return launch_peer_barrier(local_signals, peer_signals, rank, world, 0, timeout_us, *dev,
                             static_cast<cudaStream_t>(stream), epoch_counter);
}

int32_t kf_gemv(int32_t dtype, const void* x, int64_t sx_m, int64_t sx_k, const void* w,
                int64_t sw_n, int64_t sw_k, void* y, int64_t sy_m, int64_t sy_n, int64_t M,
                int64_t N, int64_t K, const kf_gemm_config* cfg, void* workspace,
                int64_t workspace_bytes, void* stream) {
  if (M > 256) return set_error(KF_ERR_UNSUPPORTED, "kf_gemv takes M <= 256; use kf_gemm");
  kf_gemm_config c = cfg ? *cfg : zero_config();
  // Up to 32 rows of x with K-contiguous 16-bit weight rows: 16-row weight
  // tiles streamed by warps straight into mma.sync fragments (measured on
  // B200 at 11008 x 4096: 0.80 of the copy bandwidth at M = 1 and 4, 0.71 at
  // M = 16, against 0.53 for 128-row TMA tiles).
  if (c.kernel == KF_GEMM_AUTO && M >= 1 && M <= GEMV_STREAM_MAX_M && N >= 1 && x != nullptr &&
      w != nullptr && y != nullptr && gemv_stream_supported(dtype, x, sx_m, sx_k, w, sw_n, sw_k, M, N, K, nullptr)) {
    int device = 0;
    int rc = current_device(&device);
    if (rc != KF_OK) return rc;
    DeviceInfo* dev = nullptr;
    rc = device_info(device, &dev);
    if (rc != KF_OK) return rc;
    if (gemv_stream_preferred(M, N, K, dev->sm_count, c.overlap != 0)) c.kernel = KF_GEMM_TILE_STREAM;
  }
  if (c.kernel == KF_GEMM_AUTO && M >= 1 && M <= GEMV_MMA_MAX_M && x != nullptr && w != nullptr &&
      y != nullptr && gemv_mma_supported(dtype, x, sx_m, sx_k, w, sw_n, sw_k, M, N, K, nullptr))
    c.kernel = KF_GEMM_TILE_ROWS;
  if (c.kernel == KF_GEMM_TILE_STREAM) {
    if (!valid_dtype(dtype)) return set_error(KF_ERR_INVALID_ARGUMENT, "unknown dtype code");
    if (M < 0 || N < 0 || K < 0) return set_error(KF_ERR_INVALID_ARGUMENT, "negative size");
    if (M == 0 || N == 0) return KF_OK;
    if (x == nullptr || w == nullptr || y == nullptr)
      return set_error(KF_ERR_INVALID_ARGUMENT, "null pointer");
    std::string why;
    if (!gemv_stream_supported(dtype, x, sx_m, sx_k, w, sw_n, sw_k, M, N, K, &why))
      return set_error(M > GEMV_STREAM_MAX_M ? KF_ERR_UNSUPPORTED : KF_ERR_UNALIGNED, "streamed tile GEMV: " + why);
    int device = 0;
    int rc = current_device(&device);
    if (rc != KF_OK) return rc;
    DeviceInfo* dev = nullptr;
    rc = device_info(device, &dev);
    if (rc != KF_OK) return rc;
    return launch_gemv_stream(dtype, x, sx_m, w, sw_n, y, sy_m, sy_n, M, N, K, c, *dev,
                              static_cast<cudaStream_t>(stream));
  }
  if (c.kernel == KF_GEMM_TILE_ROWS) {
    if (!valid_dtype(dtype)) return set_error(KF_ERR_INVALID_ARGUMENT, "unknown dtype code");
    if (M < 0 || N < 0 || K < 0) return set_error(KF_ERR_INVALID_ARGUMENT, "negative size");
    if (M == 0 || N == 0) return KF_OK;
    if (x == nullptr || w == nullptr || y == nullptr)
      return set_error(KF_ERR_INVALID_ARGUMENT, "null pointer");
    std::string why;
    if (!gemv_mma_supported(dtype, x, sx_m, sx_k, w, sw_n, sw_k, M, N, K, &why))
      return set_error(KF_ERR_UNALIGNED, "tile GEMV: " + why);
    return launch_gemv_mma(dtype, x, sx_m, w, sw_n, y, sy_m, sy_n, M, N, K, c,
                           static_cast<cudaStream_t>(stream));
  }
  if ((c.kernel == KF_GEMM_AUTO && M <= GEMV_ROWS_AUTO_MAX_M) || c.kernel == KF_GEMM_WARP_ROWS) {
    // Few rows with K-contiguous weight rows: stream the rows warp by warp on
    // CUDA cores (measured on B200: 128-row TMA tiles of a row-major weight
    // read it well below the rate a contiguous row stream reaches).
    if (!valid_dtype(dtype)) return set_error(KF_ERR_INVALID_ARGUMENT, "unknown dtype code");
    if (M < 0 || N < 0 || K < 0) return set_error(KF_ERR_INVALID_ARGUMENT, "negative size");
    if (M == 0 || N == 0) return KF_OK;
    if (x == nullptr || w == nullptr || y == nullptr)
      return set_error(KF_ERR_INVALID_ARGUMENT, "null pointer");
    int device = 0;
    int rc = current_device(&device);
    if (rc != KF_OK) return rc;
    DeviceInfo* dev = nullptr;
    rc = device_info(device, &dev);
    if (rc != KF_OK) return rc;
    std::string why;
    if (gemv_rows_supported(dtype, w, sw_n, sw_k, M, N, K, dev->max_smem_optin, &why))
      return launch_gemv_rows(dtype, x, sx_m, sx_k, w, sw_n, y, sy_m, sy_n, M, N, K, c, *dev,
                              static_cast<cudaStream_t>(stream));
    if (c.kernel == KF_GEMM_WARP_ROWS) return set_error(KF_ERR_UNALIGNED, "warp-per-row GEMV: " + why);
  }
  if (c.kernel == KF_GEMM_AUTO || c.kernel == KF_GEMM_TCGEN05) {
    if (c.swap_ab == 0) c.swap_ab = 1;
    if (c.stream_k == 0) c.stream_k = 1;
  }
  return kf_gemm(dtype, x, sx_m, sx_k, w, sw_k, sw_n, y, sy_m, sy_n, M, N, K, &c, workspace,
                 workspace_bytes, stream);
}

int64_t kf_gemm_workspace_bytes(int32_t device, int32_t dtype, int64_t sa_m, int64_t sa_k,
                                int64_t sb_k, int64_t sb_n, int64_t M, int64_t N, int64_t K,
                                const kf_gemm_config* cfg) {
  // Any 16-byte-aligned stand-in: only strides and sizes decide the config.
  // (and C a contiguous [M, N] at a 16-byte-aligned address)
  const void* stand_in = reinterpret_cast<const void*>(static_cast<uintptr_t>(256));
  return kf_gemm_workspace_bytes_for(device, dtype, stand_in, sa_m, sa_k, stand_in, sb_k, sb_n,
                                     const_cast<void*>(stand_in), N, 1, M, N, K, cfg);
}

int64_t kf_gemm_workspace_bytes_for(int32_t device, int32_t dtype, const void* a, int64_t sa_m, int64_t sa_k,
                                    const void* b, int64_t sb_k, int64_t sb_n, void* c, int64_t sc_m, int64_t sc_n,
                                    int64_t M, int64_t N, int64_t K, const kf_gemm_config* cfg) {
  DeviceInfo* dev = nullptr;
  const int rc = device_info(device, &dev);
  if (rc != KF_OK) return -rc;
  GemmArgs g;
  g.dtype = dtype;
  g.M = M;
  g.N = N;
  g.K = K;
  g.sa_m = sa_m;
  g.sa_k = sa_k;
  g.sb_k = sb_k;
  g.sb_n = sb_n;
  // A null pointer sizes for a 16-byte-aligned operand.
  const void* stand_in = reinterpret_cast<const void*>(static_cast<uintptr_t>(256));
  g.a = a != nullptr ? a : stand_in;
  g.b = b != nullptr ? b : stand_in;
  g.c = c != nullptr ? c : const_cast<void*>(stand_in);
  g.sc_m = c != nullptr ? sc_m : N;
  g.sc_n = c != nullptr ? sc_n : 1;
  const int kernel = cfg ? cfg->kernel : KF_GEMM_AUTO;
  if (kernel == KF_GEMM_TILE_STREAM) return 0;
  if ((kernel == KF_GEMM_AUTO || kernel == KF_GEMM_COLUMNS) &&
      gemv_cols_supported(dtype, g.a, g.b, sb_k, sb_n, M, N, K, nullptr))
    return gemv_cols_workspace_bytes(dtype, M, N, K, dev->sm_count);
  TcPlan plan;
  if (!plan_tc(g, cfg, *dev, -1, &plan)) return 0;
  return plan.need();
}

int64_t kf_gemv_workspace_bytes(int32_t device, int32_t dtype, int64_t sx_m, int64_t sx_k,
                                int64_t sw_n, int64_t sw_k, int64_t M, int64_t N, int64_t K,
                                const kf_gemm_config* cfg) {
  kf_gemm_config c = cfg ? *cfg : zero_config();
  // The warp-per-row kernel needs none; AUTO reports the stream-K size, since
  // a weight pointer off the 16-byte grid sends the call there.
  if (c.kernel == KF_GEMM_WARP_ROWS || c.kernel == KF_GEMM_TILE_ROWS || c.kernel == KF_GEMM_TILE_STREAM) return 0;
  if (c.kernel == KF_GEMM_AUTO || c.kernel == KF_GEMM_TCGEN05) {
    if (c.swap_ab == 0) c.swap_ab = 1;
    if (c.stream_k == 0) c.stream_k = 1;
  }
  return kf_gemm_workspace_bytes(device, dtype, sx_m, sx_k, sw_k, sw_n, M, N, K, &c);
}

int32_t kf_query_gemm_config(int32_t dtype, const kf_gemm_config* cfg, int64_t* smem_bytes,
                             int32_t* tmem_cols) {
  if (cfg == nullptr) return set_error(KF_ERR_INVALID_ARGUMENT, "null config");
  if (cfg->kernel == KF_GEMM_WARP_ROWS || cfg->kernel == KF_GEMM_TILE_ROWS ||
      cfg->kernel == KF_GEMM_TILE_STREAM) {  // no TMEM; tiny or M/K-dependent smem
    if (smem_bytes) *smem_bytes = 0;
    if (tmem_cols) *tmem_cols = 0;
    return KF_OK;
  }
  if (cfg->kernel == KF_GEMM_SIMT) {
    if (smem_bytes) *smem_bytes = 2LL * cfg->block_k * (cfg->block_m + cfg->block_n) * 4;
    if (tmem_cols) *tmem_cols = 0;
    return KF_OK;
  }
  kf_gemm_config c = *cfg;
  if (c.group_m == 0) c.group_m = 8;  // zero selects the default, as at launch
  return query_tcgen05_config(dtype, c, smem_bytes, tmem_cols);
}

int32_t kf_softmax_rows(int32_t dtype, const void* x, int64_t sx_row, void* y, int64_t sy_row,
                        int64_t rows, int64_t cols, const kf_rows_config* cfg, void* stream) {
  if (!valid_dtype(dtype)) return set_error(KF_ERR_INVALID_ARGUMENT, "unknown dtype code");
  if (rows < 0 || cols < 0) return set_error(KF_ERR_INVALID_ARGUMENT, "negative size");
  if (rows == 0 || cols == 0) return KF_OK;
  if (x == nullptr || y == nullptr) return set_error(KF_ERR_INVALID_ARGUMENT, "null pointer");
  int device = 0;
  int rc = current_device(&device);
  if (rc != KF_OK) return rc;
  DeviceInfo* dev = nullptr;
  rc = device_info(device, &dev);
  if (rc != KF_OK) return rc;
  RowsArgs a;
  a.dtype = dtype;
  a.op = 0;
  a.x = x;
  a.sx = sx_row;
  a.y = y;
  a.sy = sy_row;
  a.rows = rows;
  a.cols = cols;
  const kf_rows_config c = resolve_rows_config(a, cfg, *dev);
  return launch_rows(a, c, *dev, static_cast<cudaStream_t>(stream));
}

int32_t kf_rmsnorm_rows(int32_t dtype, const void* x, int64_t sx_row, const void* gamma,
                        void* y, int64_t sy_row, int64_t rows, int64_t cols, float eps,
                        const kf_rows_config* cfg, void* stream) {
  if (!valid_dtype(dtype)) return set_error(KF_ERR_INVALID_ARGUMENT, "unknown dtype code");
  if (rows < 0 || cols < 0) return set_error(KF_ERR_INVALID_ARGUMENT, "negative size");
  if (rows == 0 || cols == 0) return KF_OK;
  if (x == nullptr || y == nullptr || gamma == nullptr)
    return set_error(KF_ERR_INVALID_ARGUMENT, "null pointer");
  int device = 0;
  int rc = current_device(&device);
  if (rc != KF_OK) return rc;
  DeviceInfo* dev = nullptr;
  rc = device_info(device, &dev);
  if (rc != KF_OK) return rc;
  RowsArgs a;
  a.dtype = dtype;
  a.op = 1;
  a.x = x;
  a.sx = sx_row;
  a.gamma = gamma;
  a.y = y;
  a.sy = sy_row;
  a.rows = rows;
  a.cols = cols;
  a.eps = eps;
  const kf_rows_config c = resolve_rows_config(a, cfg, *dev);
  return launch_rows(a, c, *dev, static_cast<cudaStream_t>(stream));
}

int32_t kf_selftest_bounded_wait(int32_t timeout_us, void* stream) {
  if (timeout_us <= 0 || timeout_us > 5000000)
    return set_error(KF_ERR_INVALID_ARGUMENT, "timeout_us must be in (0, 5e6]");
  int device = 0;
  int rc = current_device(&device);
  if (rc != KF_OK) return rc;
  DeviceInfo* dev = nullptr;
  rc = device_info(device, &dev);
  if (rc != KF_OK) return rc;
  selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      dev->status, static_cast<unsigned long long>(timeout_us) * 1000ull);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return cuda_error(err, "launch(selftest)");
  return KF_OK;
}

}  // extern "C"
