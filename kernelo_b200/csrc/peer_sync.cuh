// Device side of the bounded cross-GPU barrier that completes an all-gather:
// shared by the stand-alone barrier kernel (peer_sync.cu) and the tile GEMV,
// whose last CTA runs it in-kernel (gemv_mma.cu).
//
// Lane t < n_peers owns peer t. It writes `epoch` into this rank's slot of
// that peer's signal array with a release store at system scope (cumulative
// over this GPU's stores into the peers' buffers that happen before it),
// then polls this rank's own slot for that peer with
// acquire loads at system scope until it reads `epoch` or a later one. The
// wait is bounded by %globaltimer: on timeout it records KF_ERR_TIMEOUT |
// SITE_PEER_BARRIER << 8 in the device status word and returns.
#pragma once

#include "kf_common.cuh"

namespace kf {

struct PeerSignals {
  uint32_t* local;                // this rank's signal array [world]
  uint32_t* peers[KF_MAX_PEERS];  // the other ranks' arrays, in rank order
  int peer_rank[KF_MAX_PEERS];    // their ranks
  int rank, n_peers;
  unsigned long long timeout_ns;
};

__device__ __forceinline__ void st_release_sys(uint32_t* addr, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* addr) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

// A peer that saw this rank's signal may run ahead and write epoch + 1 before
// this poll reads epoch, so "reached" is a wrap-safe v >= epoch.
__device__ __forceinline__ bool epoch_reached(uint32_t v, uint32_t epoch) {
  return static_cast<int32_t>(v - epoch) >= 0;
}

// Host: fill `out` from a rank's signal pointers (peers in rank order, this
// rank skipped); KF_ERR_INVALID_ARGUMENT on a null peer pointer.
int fill_peer_signals(uint32_t* local, uint32_t* const* peers, int rank, int world, int timeout_us,
                      PeerSignals* out);

// Lane t < s.n_peers signals peer t and waits for it (see above). The
// release store at system scope is the fence: it orders every write this
// lane has observed (this GPU's stores into the peers' buffers, through the
// kernel boundary or the arrival atomic) before the signal.
__device__ __forceinline__ void peer_signal_and_wait(const PeerSignals& s, uint32_t epoch, int t, int* status) {
  if (t >= s.n_peers) return;
  st_release_sys(s.peers[t] + s.rank, epoch);
  const uint32_t* mine = s.local + s.peer_rank[t];
  if (epoch_reached(ld_acquire_sys(mine), epoch)) return;
  const unsigned long long start = global_timer_ns();
  for (uint32_t spin = 1;; ++spin) {
    if (epoch_reached(ld_acquire_sys(mine), epoch)) return;
    if ((spin & 63u) == 0 && global_timer_ns() - start > s.timeout_ns) {
      record_status(status, KF_ERR_TIMEOUT, SITE_PEER_BARRIER);
      return;
    }
  }
}

}  // namespace kf
