// kf_gemv_noalloc: the decode-shape GEMV for callers that cannot allocate
// device memory.
//
// kf_gemv splits K across every SM (stream-K) and needs a few MiB of scratch
// for the fp32 partial tiles and the per-tile arrival counters; normally the
// caller passes that workspace in. Some callers have no way to do so: a plugin
// embedded in a host application that owns every device allocation (an
// inference server's memory arena, a database or engine extension) and hands
// the plugin neither an allocator nor a workspace, or a latency-critical path
// that cannot afford cudaMalloc/cudaFree, which may synchronise the device.
// For them this entry point keeps its scratch in a file-scope __device__ array
// that is part of the loaded library: KF_NOALLOC_SCRATCH_BYTES (4 MiB) on
// every GPU that loads the library, held until the process exits.
//
// Limits and behaviour:
//  - M <= KF_NOALLOC_MAX_ROWS (16); larger requests are rejected with
//    KF_ERR_WORKSPACE before anything is launched.
//  - Nothing here calls cudaMalloc, cudaFree or any allocating routine. The
//    array's device address is looked up with cudaGetSymbolAddress once per
//    device, by the first call made while that device is current; make that
//    first call before any stream capture begins.
//  - It accepts what kf_gemv accepts at M <= 16. fp16/bf16 operands with
//    K-contiguous rows (and K % 8 == 0) go to the register-fed 16-row tile
//    GEMV, which uses no scratch and never touches the array (kf_gemv's
//    default there, except beyond 8 rows at long K or many tiles, where
//    kf_gemv streams the tiles through shared memory instead).
//    The rest may take the stream-K tcgen05 GEMV (the only kernel here that
//    needs scratch) or a scratch-free CUDA-core kernel; a call whose
//    stream-K scratch would exceed the array is rejected with
//    KF_ERR_WORKSPACE before anything is launched.
//  - All calls on a device share the one array. A call that may use it
//    clears the arrival counters (cudaMemsetAsync on the caller's stream)
//    before its kernel, and the partial tiles are always written before they
//    are read. Such calls that overlap on the GPU (different streams, no
//    ordering between them) race on the array and must not be issued.
#include <mutex>
#include <string>

#include "kf_common.cuh"
#include "kf_internal.h"

namespace {

// The scratch: arrival counters first (the layout kf_gemv's stream-K kernel
// expects of any workspace), then the fp32 partial tiles.
static __device__ __align__(256) unsigned char kf_noalloc_scratch[KF_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
static_assert(kf::SK_COUNTER_BYTES <= KF_NOALLOC_SCRATCH_BYTES,
              "the stream-K counters must fit in the no-alloc scratch");

std::mutex g_scratch_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of this device's scratch array (looked up once, then cached).
int scratch_address(int device, void** out) {
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[device] == nullptr) {
    void* ptr = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&ptr, kf_noalloc_scratch);
    if (err != cudaSuccess) return kf::cuda_error(err, "cudaGetSymbolAddress(no-alloc scratch)");
    g_scratch_ptr[device] = ptr;
  }
  *out = g_scratch_ptr[device];
  return KF_OK;
}

}  // namespace

extern "C" KF_API int32_t kf_gemv_noalloc(int32_t dtype, const void* x, int64_t sx_m, int64_t sx_k,
                                          const void* w, int64_t sw_n, int64_t sw_k, void* y,
                                          int64_t sy_m, int64_t sy_n, int64_t M, int64_t N,
                                          int64_t K, void* stream) {
  if (M < 0 || N < 0 || K < 0) return kf::set_error(KF_ERR_INVALID_ARGUMENT, "negative size");
  if (M > KF_NOALLOC_MAX_ROWS)
    return kf::set_error(KF_ERR_WORKSPACE,
                         "kf_gemv_noalloc takes at most " + std::to_string(KF_NOALLOC_MAX_ROWS) +
                             " rows (M=" + std::to_string(M) +
                             "): its scratch is a fixed " +
                             std::to_string(KF_NOALLOC_SCRATCH_BYTES) + "-byte array");
  if (M == 0 || N == 0) return KF_OK;
  int device = 0;
  int rc = kf::current_device(&device);
  if (rc != KF_OK) return rc;
  if (device >= kMaxDevices) return kf::set_error(KF_ERR_INVALID_ARGUMENT, "device index out of range");
  // K-contiguous 16-bit operands take the 16-row tile kernel, which needs no
  // scratch at all (and so cannot race with an overlapping call). The rest go
  // through kf_gemv's own choice (the default config): the stream-K tcgen05
  // GEMV, the one kernel whose scratch this entry point holds, or a
  // scratch-free CUDA-core kernel for operands TMA cannot describe.
  if (x != nullptr && w != nullptr && y != nullptr &&
      kf::gemv_mma_supported(dtype, x, sx_m, sx_k, w, sw_n, sw_k, M, N, K, nullptr))
    return kf::launch_gemv_mma(dtype, x, sx_m, w, sw_n, y, sy_m, sy_n, M, N, K, kf_gemm_config{},
                               static_cast<cudaStream_t>(stream));
  kf_gemm_config cfg{};  // KF_GEMM_AUTO, as kf_gemv(..., cfg = NULL)
  const int64_t need = kf_gemv_workspace_bytes(device, dtype, sx_m, sx_k, sw_n, sw_k, M, N, K, &cfg);
  if (need < 0) return static_cast<int32_t>(-need);
  if (need > KF_NOALLOC_SCRATCH_BYTES)
    return kf::set_error(KF_ERR_WORKSPACE, "this GEMV needs " + std::to_string(need) +
                                               " bytes of scratch, above the fixed " +
                                               std::to_string(KF_NOALLOC_SCRATCH_BYTES));
  void* scratch = nullptr;
  rc = scratch_address(device, &scratch);
  if (rc != KF_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (need > 0) {
    // The arrival counters must start at zero; the array keeps whatever the
    // previous call (or an aborted one) left.
    const cudaError_t err = cudaMemsetAsync(scratch, 0, kf::SK_COUNTER_BYTES, s);
    if (err != cudaSuccess) return kf::cuda_error(err, "cudaMemsetAsync(no-alloc counters)");
  }
  return kf_gemv(dtype, x, sx_m, sx_k, w, sw_n, sw_k, y, sy_m, sy_n, M, N, K, &cfg, scratch,
                 KF_NOALLOC_SCRATCH_BYTES, stream);
}
