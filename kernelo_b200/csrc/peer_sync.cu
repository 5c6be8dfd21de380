// Cross-GPU barrier over peer-mapped signal words (sm_100a), for the
// all-gathering fused linear: after every rank's GEMM has stored its output
// tiles into all peers' copies of Y, this publishes "my stores are done" and
// waits for the same from every peer.
//
// One warp: lane t < world - 1 owns peer t. It writes `epoch` into the slot
// of this rank in that peer's signal array with a release store at system
// scope, then polls this rank's own slot for that peer with acquire loads at
// system scope until it reads `epoch` or a later one. The GEMM or GEMV that
// stored into the peers precedes this kernel on the stream and has completed
// when it starts; the system-scope fence before the release store is
// cumulative over those stores, so a peer that observes the signal also
// observes the data. Every wait is bounded by
// %globaltimer: on timeout the kernel records
// KF_ERR_TIMEOUT | SITE_PEER_BARRIER << 8 in the device status word and
// returns, leaving the context usable.
//
// The counted form keeps the epoch in a device word of this rank: the kernel
// takes *counter + 1 and stores it back, so a captured CUDA graph that holds
// the barrier advances the epoch on every replay (a host-supplied epoch would
// be frozen into the graph and let later replays pass unsynchronised).
#include <cuda.h>

#include <cstring>
#include <mutex>

#include "kf_common.cuh"
#include "kf_internal.h"
#include "peer_sync.cuh"

namespace kf {
namespace {

struct PeerBarrierParams {
  PeerSignals sig;
  uint32_t epoch;
  uint32_t* counter;  // counted form: the epoch is *counter + 1 (this rank's memory)
  int* status;
};

__global__ void peer_barrier_kernel(const PeerBarrierParams p) {
  const int t = threadIdx.x;
  uint32_t epoch = p.epoch;
  if (p.counter != nullptr) {
    // Every lane reads the previous epoch before lane 0 advances it; the
    // previous barrier on this stream wrote it (kernel boundary).
    epoch = *p.counter + 1u;
    __syncwarp();
    if (t == 0) *p.counter = epoch;
  }
  peer_signal_and_wait(p.sig, epoch, t, p.status);
}

}  // namespace

int fill_peer_signals(uint32_t* local, uint32_t* const* peers, int rank, int world, int timeout_us,
                      PeerSignals* out) {
  PeerSignals& s = *out;
  s.local = local;
  s.rank = rank;
  s.n_peers = world - 1;
  for (int i = 0, r = 0; r < world; ++r) {
    if (r == rank) continue;
    if (peers[i] == nullptr) return set_error(KF_ERR_INVALID_ARGUMENT, "null peer signal pointer");
    s.peers[i] = peers[i];
    s.peer_rank[i] = r;
    ++i;
  }
  s.timeout_ns = static_cast<unsigned long long>(timeout_us) * 1000ull;
  return KF_OK;
}

int launch_peer_barrier(uint32_t* local, uint32_t* const* peers, int rank, int world,
                        uint32_t epoch, int timeout_us, const DeviceInfo& dev, cudaStream_t stream,
                        uint32_t* counter) {
  if (world < 1 || world > KF_MAX_PEERS + 1)
    return set_error(KF_ERR_INVALID_ARGUMENT, "world must be in [1, 8]");
  if (rank < 0 || rank >= world) return set_error(KF_ERR_INVALID_ARGUMENT, "rank out of range");
  if (timeout_us <= 0 || timeout_us > 60000000)
    return set_error(KF_ERR_INVALID_ARGUMENT, "timeout_us must be in (0, 6e7]");
  if (counter == nullptr && epoch == 0)
    return set_error(KF_ERR_INVALID_ARGUMENT, "epochs start at 1 (0 is the initial value)");
  if (world == 1) return KF_OK;
  if (local == nullptr || peers == nullptr)
    return set_error(KF_ERR_INVALID_ARGUMENT, "null signal pointer");
  PeerBarrierParams p{};
  const int rc = fill_peer_signals(local, peers, rank, world, timeout_us, &p.sig);
  if (rc != KF_OK) return rc;
  p.epoch = epoch;
  p.counter = counter;
  p.status = dev.status;
  peer_barrier_kernel<<<1, 32, 0, stream>>>(p);
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return cuda_error(err, "launch(peer barrier)");
  return KF_OK;
}

// ------------------------------------------------------------------ IPC mapping
// Peer copies of a buffer are mapped with CUDA IPC handles (no multicast
// object is ever created). A handle names a whole allocation, so the exporter
// also reports where its pointer sits inside it (allocators sub-allocate).

namespace {
using AddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

AddressRangeFn address_range_fn() {
  static AddressRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* sym = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &sym, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddressRangeFn>(sym);
  });
  return fn;
}
}  // namespace

}  // namespace kf

using namespace kf;

int32_t kf_ipc_handle(const void* ptr, void* handle_out, int64_t* offset_out) {
  if (ptr == nullptr || handle_out == nullptr || offset_out == nullptr)
    return set_error(KF_ERR_INVALID_ARGUMENT, "null pointer");
  AddressRangeFn range = address_range_fn();
  if (range == nullptr) return set_error(KF_ERR_NO_DEVICE, "cuMemGetAddressRange is not available");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return set_error(KF_ERR_INVALID_ARGUMENT, "pointer is not device memory of this process");
  cudaIpcMemHandle_t h;
  const cudaError_t err = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (err != cudaSuccess) return cuda_error(err, "cudaIpcGetMemHandle");
  static_assert(sizeof(h) == KF_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return KF_OK;
}

int32_t kf_ipc_open(const void* handle, void** base_out) {
  if (handle == nullptr || base_out == nullptr) return set_error(KF_ERR_INVALID_ARGUMENT, "null pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  const cudaError_t err = cudaIpcOpenMemHandle(base_out, h, cudaIpcMemLazyEnablePeerAccess);
  if (err != cudaSuccess) return cuda_error(err, "cudaIpcOpenMemHandle");
  return KF_OK;
}

int32_t kf_ipc_close(void* base) {
  if (base == nullptr) return set_error(KF_ERR_INVALID_ARGUMENT, "null pointer");
  const cudaError_t err = cudaIpcCloseMemHandle(base);
  if (err != cudaSuccess) return cuda_error(err, "cudaIpcCloseMemHandle");
  return KF_OK;
}
