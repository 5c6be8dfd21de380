// Host-side declarations shared by the translation units of libkernelo_b200.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "kernelo_b200.h"

namespace kf {

// Records the message returned by kf_last_error() and passes the code through.
int set_error(int code, const std::string& message);
int cuda_error(cudaError_t err, const char* where);

// Per-device facts, cached on first use.
struct DeviceInfo {
  int sm_count = 0;
  int max_smem_optin = 0;
  int major = 0;
  int minor = 0;
  int* status = nullptr;  // device address of this device's status word
};
int device_info(int device, DeviceInfo** out);
int current_device(int* device);

// One GEMM problem as the C ABI received it (element strides).
struct GemmArgs {
  int dtype = KF_FP16;
  const void* a = nullptr;
  int64_t sa_m = 0, sa_k = 0;
  const void* b = nullptr;
  int64_t sb_k = 0, sb_n = 0;
  void* c = nullptr;
  int64_t sc_m = 0, sc_n = 0;
  int64_t M = 0, N = 0, K = 0;
  const void* bias = nullptr;
  int epilogue = KF_EPI_NONE;
  void* workspace = nullptr;
  int64_t workspace_bytes = 0;
  // Peer copies of C (device pointers to the same element (0, 0) in other
  // GPUs' buffers of the same layout): the epilogue stores every output tile
  // into each of them as well (the all-gather of a column-sharded linear).
  void* peers[KF_MAX_PEERS] = {};
  int n_peers = 0;
  // fp32 only: a and b are TF32-split operands (tf32_split.cu), K-major rows
  // of [small | big] with K (= kp) elements each; the tcgen05 kernel runs
  // them as kind::tf32, three MMAs per k-block.
  bool tf32_split = false;
  // Peer barrier to run after the all-gather (kf_linear_bias_act_allgather_sync):
  // the tile GEMV runs it in its last CTA and sets sync_done.
  const kf_peer_sync* sync = nullptr;
  bool sync_done = false;
};

// Stream-K workspace layout (tcgen05 GEMM): one int32 arrival counter per
// output tile first, at a fixed offset, then the fp32 partial tiles.
constexpr int64_t SK_MAX_TILES = 16384;
constexpr int64_t SK_COUNTER_BYTES = SK_MAX_TILES * 4;

// Fills zero fields of `cfg` with the library default for this problem.
kf_gemm_config resolve_gemm_config(const GemmArgs& args, const kf_gemm_config* user,
                                   int sm_count);

// tcgen05 path. Returns KF_ERR_UNALIGNED when the operands cannot be described
// by TMA tensor maps, KF_ERR_INVALID_CONFIG for configs the kernel cannot run.
int launch_gemm_tcgen05(const GemmArgs& args, const kf_gemm_config& cfg, const DeviceInfo& dev,
                        cudaStream_t stream);
int64_t gemm_tcgen05_workspace_bytes(const GemmArgs& args, const kf_gemm_config& cfg,
                                     const DeviceInfo& dev);
int query_tcgen05_config(int dtype, const kf_gemm_config& cfg, int64_t* smem_bytes,
                         int32_t* tmem_cols);
// Whether the operands can take the tcgen05 path (TMA strides/alignment).
bool tcgen05_operands_ok(const GemmArgs& args, std::string* why);
// Whether one operand (element strides along its M/N and K extents) can be
// described by a TMA tensor map: 16-byte base, unit stride along K or M/N,
// the other stride a multiple of 8 elements, K >= 8.
bool tma_describable(const void* ptr, int64_t s_mn, int64_t s_k, int64_t mn, int64_t k);

// Operand packing (pack.cu): a 16-bit operand TMA cannot describe, copied
// into the workspace as a pitched matrix the tcgen05 kernel can read.
struct PackedOperand {
  bool k_inner = true;      // K is the copy's inner (unit-stride) dimension
  int64_t outer = 0;        // rows of the copy (the padded K when MN is inner)
  int64_t src_outer = 0;    // rows that exist in the source
  int64_t len = 0;          // elements per source row
  int64_t pitch = 0;        // elements per row of the copy (a multiple of 8)
  int64_t bytes = 0;        // size of the copy, 256-byte rounded
  const void* src = nullptr;
  int64_t s_outer = 0, s_inner = 0;
};
// The copy of an operand with element strides (s_mn, s_k) and extents
// (mn, k); K is padded with zero rows/columns to k_padded (>= k).
PackedOperand plan_pack(const void* ptr, int64_t s_mn, int64_t s_k, int64_t mn, int64_t k, int64_t k_padded);
int launch_pack(const PackedOperand& p, void* dst, cudaStream_t stream);
// An output C [m, n] whose rows are off the 16-byte grid, staged as a pitched
// copy: the GEMM writes the copy with vector stores, launch_unpack moves it to C.
PackedOperand plan_output_stage(void* c, int64_t sc_m, int64_t sc_n, int64_t m, int64_t n);
int launch_unpack(const PackedOperand& p, const void* staged, cudaStream_t stream);

// fp32 operands split for 3xTF32 (tf32_split.cu): rows of [small|big] TF32
// parts, K padded with zeros to kp (a multiple of 32), written K-major with
// `pitch` = 2 kp elements. (s_r, s_k): the source's element strides of (row, k).
struct SplitOperand {
  const void* src = nullptr;
  int64_t s_r = 0, s_k = 0;
  int64_t rows = 0, K = 0, kp = 0, pitch = 0;
  int64_t bytes = 0;  // 256-byte rounded
};
SplitOperand plan_tf32_split(const void* src, int64_t s_r, int64_t s_k, int64_t rows, int64_t K);
int launch_tf32_split(const SplitOperand& s, void* dst, cudaStream_t stream);

// CUDA-core path: any strides, fp16/bf16/fp32.
int launch_gemm_simt(const GemmArgs& args, const kf_gemm_config& cfg, cudaStream_t stream);

// Warp-per-row decode GEMV (gemv_rows.cu): y[M, N] = x[M, K] . w[N, K]^T for
// M <= GEMV_ROWS_MAX_M with K-contiguous, 16-byte-aligned weight rows.
// Shared memory the all-gathering GEMM epilogue stages its output in: per
// epilogue warp, 32 rows x 64 columns of 2-byte elements, 1024-byte aligned
// (the 128-byte swizzle of a TMA box repeats every 8 rows).
constexpr int GEMM_PEER_STAGE_BYTES = 8 * 32 * 64 * 2;
constexpr int GEMM_PEER_STAGE_SMEM = GEMM_PEER_STAGE_BYTES + 1024;

// 16-row tile decode GEMV (gemv_mma.cu): M <= 32, fp16/bf16. With n_peers > 0
// every output element is also stored at the same offset from each peers[i]
// (the decode-shape all-gather; the caller's barrier publishes it).
constexpr int GEMV_MMA_MAX_M = 32;
bool gemv_mma_supported(int dtype, const void* x, int64_t sx_m, int64_t sx_k, const void* w, int64_t sw_n,
                        int64_t sw_k, int64_t M, int64_t N, int64_t K, std::string* why);
int launch_gemv_mma(int dtype, const void* x, int64_t sx_m, const void* w, int64_t sw_n, void* y,
                    int64_t sy_m, int64_t sy_n, int64_t M, int64_t N, int64_t K,
                    const kf_gemm_config& cfg, cudaStream_t stream, int epilogue = KF_EPI_NONE,
                    const void* bias = nullptr, void* const* peers = nullptr, int n_peers = 0,
                    const kf_peer_sync* sync = nullptr, int* status = nullptr);

// Streamed 16-row tile decode GEMV (gemv_stream.cu): M <= 16, fp16/bf16, the
// tile kernel's operand rules; one persistent CTA per SM streams its tiles
// through a shared-memory ring of bulk copies. No peers, no workspace.
constexpr int GEMV_STREAM_MAX_M = 16;
constexpr int GEMV_STREAM_DEFAULT_CHUNK = 1024;  // weight elements per row per stage
bool gemv_stream_supported(int dtype, const void* x, int64_t sx_m, int64_t sx_k, const void* w, int64_t sw_n,
                           int64_t sw_k, int64_t M, int64_t N, int64_t K, std::string* why);
// The library's choice of the streamed kernel over the register-fed one for a
// supported decode shape (measured on B200, graph-timed back-to-back
// launches). Without overlap: beyond 8 rows of x when K is long or the 16-row
// tiles number at least eight per SM (16 x 4096 x 11008: 20.9 us against
// 26.9; 16 x 44032 x 4096: 63.6 against 66.5). With overlap (only the streamed
// kernel prefetches its weight while the previous grid finishes) also beyond
// 8 rows at any N (16 x 11008 x 4096: 17.8-18.2 us against 18.3), for long K
// at any M (4 x 4096 x 11008: 17.6 against 20.2) and below four tiles per SM;
// up to 8 rows on many tiles of short K the register-fed kernel in stream
// order stays ahead (1 x 11008 x 4096: 15.1-15.4 us against 15.3-17.3).
inline bool gemv_stream_preferred(int64_t M, int64_t N, int64_t K, int sm_count, bool overlap) {
  if (M < 1 || M > GEMV_STREAM_MAX_M) return false;
  const int64_t tiles = (N + 15) / 16;
  if (overlap) return M > 8 || K >= 8192 || tiles < 4LL * sm_count;
  return M > 8 && (K >= 8192 || tiles >= 8LL * sm_count);
}
int launch_gemv_stream(int dtype, const void* x, int64_t sx_m, const void* w, int64_t sw_n, void* y,
                       int64_t sy_m, int64_t sy_n, int64_t M, int64_t N, int64_t K, const kf_gemm_config& cfg,
                       const DeviceInfo& dev, cudaStream_t stream, int epilogue = KF_EPI_NONE,
                       const void* bias = nullptr);

// Decode-shape GEMM against an N-contiguous B (gemv_cols.cu): M <= 8, any
// dtype, K split over CTAs with a deterministic last-arrival sum.
constexpr int GEMV_COLS_MAX_M = 8;
bool gemv_cols_supported(int dtype, const void* x, const void* b, int64_t sb_k, int64_t sb_n, int64_t M,
                         int64_t N, int64_t K, std::string* why);
int gemv_cols_splits(int dtype, int64_t M, int64_t N, int64_t K, int sm_count);
int64_t gemv_cols_workspace_bytes(int dtype, int64_t M, int64_t N, int64_t K, int sm_count);
int launch_gemv_cols(int dtype, const void* x, int64_t sx_m, int64_t sx_k, const void* b, int64_t sb_k,
                     void* y, int64_t sy_m, int64_t sy_n, int64_t M, int64_t N, int64_t K, int epilogue,
                     const void* bias, void* workspace, int64_t workspace_bytes, int sm_count,
                     cudaStream_t stream);

// Softmax kernel choice by row width in 16-byte vectors (rows.cu).
constexpr long long SOFTMAX_STREAM_MAX_VECTORS = 128;     // up to 2 KB: streaming kernel
constexpr long long SOFTMAX_REGISTER_MAX_VECTORS = 2048;  // up to 32 KB: register kernel

constexpr int GEMV_ROWS_MAX_M = 4;
// kf_gemv picks it by itself up to this many rows (measured on B200: at M=4
// the tcgen05 GEMV streams the weight faster).
constexpr int GEMV_ROWS_AUTO_MAX_M = 2;
bool gemv_rows_supported(int dtype, const void* w, int64_t sw_n, int64_t sw_k, int64_t M,
                         int64_t N, int64_t K, int max_smem_optin, std::string* why);
int launch_gemv_rows(int dtype, const void* x, int64_t sx_m, int64_t sx_k, const void* w,
                     int64_t sw_n, void* y, int64_t sy_m, int64_t sy_n, int64_t M, int64_t N,
                     int64_t K, const kf_gemm_config& cfg, const DeviceInfo& dev,
                     cudaStream_t stream);

// Cross-GPU barrier over peer-mapped signal words (peer_sync.cu).
// counter != nullptr: the epoch is *counter + 1, advanced on the device (epoch unused).
int launch_peer_barrier(uint32_t* local, uint32_t* const* peers, int rank, int world,
                        uint32_t epoch, int timeout_us, const DeviceInfo& dev, cudaStream_t stream,
                        uint32_t* counter = nullptr);

// Row kernels.
struct RowsArgs {
  int dtype = KF_FP16;
  int op = 0;  // 0 softmax, 1 rmsnorm
  const void* x = nullptr;
  int64_t sx = 0;
  const void* gamma = nullptr;
  void* y = nullptr;
  int64_t sy = 0;
  int64_t rows = 0, cols = 0;
  float eps = 0.0f;
};
// Fills zero fields of `cfg`: kernel choice (streaming for many rows whose
// x/y phases allow it), then that kernel's warps / cluster.
kf_rows_config resolve_rows_config(const RowsArgs& args, const kf_rows_config* user,
                                   const DeviceInfo& dev);
int launch_rows(const RowsArgs& args, const kf_rows_config& cfg, const DeviceInfo& dev,
                cudaStream_t stream);
// Streaming kernel (rows_stream.cu).
bool rows_stream_supported(const RowsArgs& args, int max_smem_optin, std::string* why);
// Warp-per-row persistent kernel for narrow rows (rows_warp.cu): rows of whole
// 16-byte vectors, up to 128 of them, starting on the 16-byte grid.
// Widest rows (16-byte vectors) of the warp-per-row kernel: its default for
// softmax (2 KB) and for RMSNorm (4 KB), and what it takes at all (4 KB).
constexpr long long ROWS_WARP_MAX_VECTORS = 128;
constexpr long long ROWS_WARP_RMSNORM_MAX_VECTORS = 256;
constexpr long long ROWS_WARP_EXPLICIT_MAX_VECTORS = 256;
bool rows_warp_supported(const RowsArgs& args, std::string* why);
int launch_rows_warp(const RowsArgs& args, const DeviceInfo& dev, cudaStream_t stream);
int stream_default_warps(int64_t cols, int elem);
int launch_rows_stream(const RowsArgs& args, const kf_rows_config& cfg, const DeviceInfo& dev,
                       cudaStream_t stream);

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

}  // namespace kf
