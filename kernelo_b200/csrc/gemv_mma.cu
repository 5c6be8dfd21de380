// Decode-shape GEMV with 16-row weight tiles: y[m, n] = epi(sum_k x[m, k] w[n, k])
// for M <= 32 and a weight whose rows are K-contiguous (nn.Linear's [N, K]);
// epi is none, + bias[n], or + bias[n] then GELU (the fused linear at decode
// shapes).
//
// The product is ~M FLOP per weight byte, so the kernel's job is to stream W
// from HBM at full rate; the arithmetic must only stay out of the way. One CTA
// takes one 16-row tile of W and splits its K extent over its S warps. Lane
// (g, t) (g = lane / 4, t = lane % 4) loads 16-byte vectors of weight rows g
// and g + 8 at vector positions t, t + 4, t + 8, ... of its warp's K slice, so
// each quad of lanes reads 64 contiguous bytes of a row and every row is read
// front to back. Those registers are the A fragments of `mma.sync.m16n8k16`
// as loaded: the K order inside an MMA is free as long as A and B agree, and a
// lane's B fragment is x[g (+8)][the same eight K positions], a 16-byte load
// from L1/L2 (x is a few KB). So there is no conversion, no shared-memory
// staging of x and no prologue: the first weight loads go out at once. Each
// 16-byte vector pair feeds two MMAs per 8 rows of x; products accumulate in
// fp32. The S partial tiles are summed through shared memory and rounded
// once into y.
//
// The tensor-core instruction here is the warp-level mma.sync, not tcgen05:
// at M <= 32 the contraction is a small part of the time, and what decides the
// speed is the weight stream. tcgen05 operands come from shared memory as TMA
// boxes of 128 rows x 128 bytes, which measured 3.5 TB/s on this shape; rows
// streamed contiguously by warps measured 4.8 TB/s (same W, same M).
//
// With peer pointers the kernel is also the column-sharded decode layer's
// all-gather: each output element goes to this rank's y and, at the same
// offset, to every peer's copy (at M = 16 and 8 ranks, 44 KB per peer), so
// no collective follows the GEMV -- only the bounded peer barrier.
//
// Replaces the reference's matmul launch at decode shapes
// (kernelforge/kernels/matmul.py:132-155 with M in {1, 4, 16}); fp32
// accumulation and one output rounding as in the reference's matmul.
#include <cooperative_groups.h>

#include "kf_common.cuh"
#include "kf_internal.h"
#include "peer_sync.cuh"

namespace cg = cooperative_groups;

namespace kf {
namespace {

struct GemvMmaParams {
  const void* x;
  long long sx_m;  // x rows are K-contiguous
  const void* w;
  long long sw_n;
  void* y;
  long long sy_m, sy_n;
  const void* bias;  // [N], for the bias / GELU epilogues
  int M, N, K;
  // CTAs per weight tile (a thread-block cluster along x): the tile's K extent
  // is split over ks x S warps and the CTAs' sums meet in the leader's shared
  // memory. 1 unless the tiles are too few to fill the GPU (a column shard).
  int ks;
  // Peer copies of y (same strides; the element that corresponds to y[0, 0]):
  // every output element is stored there too -- the decode-shape all-gather.
  int n_peers;
  void* peers[KF_MAX_PEERS];
  // In-kernel peer barrier (sync = 1): every storing CTA counts itself on
  // `arrivals`; the last one advances *epoch_counter and signals the peers.
  int sync;
  uint32_t* arrivals;
  uint32_t* epoch_counter;
  unsigned int storing_ctas;
  PeerSignals sig;
  int* status;
};

// NT: 8-row groups of x (1 for M <= 8, 2 for M <= 16, 4 for M <= 32); S: warps per CTA (K
// slices); U: vector pairs per lane in flight.
// At least five CTAs per SM: a tile's CTA lasts about the whole kernel, so
// all of them (688 for N = 11008) must be resident at once.
// Weight vectors bypass L1 allocation (each is read once); x vectors are kept
// in L1 ahead of other lines (every warp of every CTA on the SM re-reads them;
// load_x in kf_common.cuh).
// At M = 16 x is 128 KB per CTA, as much as the CTA's weights: without the
// hints the weight stream evicts it (39 % L1 hits measured).
__device__ __forceinline__ uint4 load_weight(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// SPLIT: compiled for a K split over a cluster (p.ks > 1); without it the
// split's index arithmetic folds away (it cost spills at 48 registers, and
// 1.6 us at N = 11008).
template <typename T, int NT, int S, int U, int EPI, bool SPLIT>
__global__ void __launch_bounds__(32 * S, 5) gemv_mma_kernel(const GemvMmaParams p) {
  __shared__ float4 part[S > 1 ? S - 1 : 1][32][NT];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int ks = SPLIT ? p.ks : 1;
  const int part_rank = static_cast<int>(blockIdx.x) % ks;  // == the rank in the cluster
  const int n0 = static_cast<int>(blockIdx.x) / ks * 16;
  const int nvec = p.K / 8;  // 16-byte vectors per row (K % 8 == 0)
  // This warp's K slice, in whole quads of vectors.
  const int quads = (nvec + 3) / 4;
  const int slice = part_rank * S + warp;  // of ks * S slices
  const int q0 = static_cast<int>(static_cast<long long>(quads) * slice / (ks * S));
  const int q1 = static_cast<int>(static_cast<long long>(quads) * (slice + 1) / (ks * S));
  const int ra = min(n0 + g, p.N - 1), rb = min(n0 + g + 8, p.N - 1);  // clamped rows are not stored
  const uint4* wa = reinterpret_cast<const uint4*>(static_cast<const T*>(p.w) + ra * p.sw_n);
  const uint4* wb = reinterpret_cast<const uint4*>(static_cast<const T*>(p.w) + rb * p.sw_n);
  const uint4* xr[NT];
  bool xon[NT];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int m = g + 8 * nt;
    xon[nt] = m < p.M;
    xr[nt] = reinterpret_cast<const uint4*>(static_cast<const T*>(p.x) + (xon[nt] ? m : 0) * p.sx_m);
  }
  float acc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[nt][i] = 0.0f;

  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
  // A batch: U vector pairs (rows g and g + 8) at quads q .. q + U - 1.
  auto load_batch = [&](int q, uint4 (&va)[U], uint4 (&vb)[U]) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int v = 4 * (q + u) + t;
      const bool ok = q + u < q1 && v < nvec;
      va[u] = ok ? load_weight(wa + v) : zero;
      vb[u] = ok ? load_weight(wb + v) : zero;
    }
  };
  // x is read per vector just before its MMAs (L1 hits), which keeps its
  // registers short-lived.
  auto mma_batch = [&](int q, const uint4 (&va)[U], const uint4 (&vb)[U]) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int v = 4 * (q + u) + t;
      const bool ok = q + u < q1 && v < nvec;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const uint4 vx = (ok && xon[nt]) ? load_x(xr[nt] + v) : zero;
        // elements 0-3 of the vector, then 4-7: logical k {2t, 2t+1, 2t+8, 2t+9}
        mma16816<T>(acc[nt], va[u].x, vb[u].x, va[u].y, vb[u].y, vx.x, vx.y);
        mma16816<T>(acc[nt], va[u].z, vb[u].z, va[u].w, vb[u].w, vx.z, vx.w);
      }
    }
  };
  if constexpr (U == 1) {
    // One pair a batch, software-pipelined: the next pair's loads go out
    // before this pair's MMAs, so a warp always has a load in flight.
    uint4 ca[1], cb[1], na[1], nb[1];
    load_batch(q0, ca, cb);
    for (int q = q0; q < q1; ++q) {
      load_batch(q + 1, na, nb);
      mma_batch(q, ca, cb);
      ca[0] = na[0];
      cb[0] = nb[0];
    }
  } else {
    // The weight loads of a batch go out together (HBM), then its MMAs.
    for (int q = q0; q < q1; q += U) {
      uint4 va[U], vb[U];
      load_batch(q, va, vb);
      mma_batch(q, va, vb);
    }
  }

  if constexpr (S > 1) {
    if (warp > 0) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
        part[warp - 1][lane][nt] = make_float4(acc[nt][0], acc[nt][1], acc[nt][2], acc[nt][3]);
    }
    __syncthreads();
    if (warp == 0) {
#pragma unroll
      for (int s = 0; s < S - 1; ++s)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const float4 o = part[s][lane][nt];
          acc[nt][0] += o.x;
          acc[nt][1] += o.y;
          acc[nt][2] += o.z;
          acc[nt][3] += o.w;
        }
    }
  }
  if constexpr (SPLIT) {
    // Across the cluster: every CTA's warp 0 leaves its sum in its own shared
    // memory; the leader adds the others' in rank order (deterministic) and
    // runs the epilogue. No thread exits before both cluster barriers.
    __shared__ float4 cta_sum[32][NT];
    cg::cluster_group cluster = cg::this_cluster();
    if (warp == 0 && part_rank != 0) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) cta_sum[lane][nt] = make_float4(acc[nt][0], acc[nt][1], acc[nt][2], acc[nt][3]);
    }
    cluster.sync();
    if (warp == 0 && part_rank == 0) {
      for (int r = 1; r < ks; ++r) {
        const float4* other = cluster.map_shared_rank(&cta_sum[0][0], static_cast<unsigned>(r));
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const float4 o = other[lane * NT + nt];
          acc[nt][0] += o.x;
          acc[nt][1] += o.y;
          acc[nt][2] += o.z;
          acc[nt][3] += o.w;
        }
      }
    }
    cluster.sync();  // the others' shared memory stays until the leader has read it
    if (part_rank != 0) return;
  }
  if (warp > 0) return;
  // D fragment: acc[nt][0..1] = rows n0+g, x rows 8nt+2t, +1; [2..3] = rows n0+g+8.
  // The fused linear's epilogue (bias[n], then GELU) runs here, before the
  // one rounding, as in the GEMM.
  T* y = static_cast<T*>(p.y);
  float bias[2] = {0.0f, 0.0f};
  if constexpr (EPI != KF_EPI_NONE) {
    const T* b = static_cast<const T*>(p.bias);
#pragma unroll
    for (int h = 0; h < 2; ++h) bias[h] = to_f32(b[min(n0 + g + 8 * h, p.N - 1)]);
  }
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int m = 8 * nt + 2 * t + (i & 1);
      const int n = n0 + g + (i >> 1) * 8;
      if (m < p.M && n < p.N) {
        const long long off = m * p.sy_m + static_cast<long long>(n) * p.sy_n;
        const T v = from_f32<T>(apply_epilogue<EPI>(acc[nt][i], bias[i >> 1]));
        y[off] = v;
        // Peer stores: the same element into every other rank's copy of y over
        // NVLink. Eight lanes of a quad column write 16 contiguous bytes.
#pragma unroll
        for (int j = 0; j < KF_MAX_PEERS; ++j)
          if (j < p.n_peers) static_cast<T*>(p.peers[j])[off] = v;
      }
    }
  }
  // No fence per CTA: the barrier fences once at system scope, cumulatively
  // over these stores. (A fence.sc.sys at the end of every CTA measured +9 us
  // on a 2-way shard of 11008 x 4096, 11 -> 20 us, with the "peer" copy in
  // local memory as much as over NVLink.) The barrier is either the kernel
  // that follows on the stream, or (sync) this kernel's last CTA: each CTA's
  // warp counts itself with an acq_rel atomic at GPU scope after its lanes'
  // stores (ordered by __syncwarp), so the last one has observed every CTA's
  // stores before it fences and signals.
  if (p.sync) {
    __syncwarp();
    unsigned int last = 0;
    if (lane == 0) {
      unsigned int prev;
      asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(prev) : "l"(p.arrivals) : "memory");
      last = prev + 1u == p.storing_ctas ? 1u : 0u;
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (last) {
      uint32_t epoch = 0;
      if (lane == 0) {
        *p.arrivals = 0u;  // for the next launch (kernel boundary)
        epoch = *p.epoch_counter + 1u;
        *p.epoch_counter = epoch;
      }
      epoch = __shfl_sync(0xffffffffu, epoch, 0);
      peer_signal_and_wait(p.sig, epoch, lane, p.status);
    }
  }
}

template <typename T, int NT, int S, int U, int EPI>
int launch_shape(const GemvMmaParams& p, cudaStream_t stream) {
  const unsigned tiles = static_cast<unsigned>((p.N + 15) / 16);
  cudaLaunchConfig_t lc{};
  lc.gridDim = dim3(tiles * static_cast<unsigned>(p.ks));
  lc.blockDim = dim3(32 * S);
  lc.stream = stream;
  cudaLaunchAttribute attr[1];
  if (p.ks > 1) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(p.ks);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
  }
  const cudaError_t err = p.ks > 1 ? cudaLaunchKernelEx(&lc, gemv_mma_kernel<T, NT, S, U, EPI, true>, p)
                                   : cudaLaunchKernelEx(&lc, gemv_mma_kernel<T, NT, S, U, EPI, false>, p);
  if (err != cudaSuccess) return cuda_error(err, "launch(gemv mma)");
  return KF_OK;
}

// CTAs per weight tile: the fewest (1, 2, 4) that give at least two CTAs per
// SM up to 8 rows of x, four beyond (a tile's CTA streams its weights for
// about the whole kernel, so too few CTAs leave HBM idle; more x rows make
// each CTA slower and want more of them). Measured on B200 at K = 4096
// (graph-timed; M = 1 / M = 16, us): N = 5504 split 1 9.9 / 14.0, split 2
// 10.9 / 13.3; N = 2752 split 2 8.1 / 10.3, split 4 7.6 / 10.1; N = 1376
// split 4 6.1 / 7.8, split 8 6.3 / 8.4.
int default_tile_split(long long tiles, int m) {
  static thread_local int cached_device = -1, sms = 148;
  int device = 0;
  if (cudaGetDevice(&device) == cudaSuccess && device != cached_device) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) == cudaSuccess && v > 0) sms = v;
    cached_device = device;
  }
  const long long target = static_cast<long long>(m <= 8 ? 2 : 4) * sms;
  int ks = 1;
  while (ks < 4 && tiles * ks < target) ks *= 2;
  return ks;
}

// Launch shapes (S warps per tile, U vector pairs per batch per lane; U = 1
// is the software-pipelined single pair): config block_m selects S and stages
// selects U; zero picks the default, measured on B200 at N = 11008, K = 4096
// (graph-timed, weights beyond L2): (8, 1) up to 8 rows of x (15.5 / 15.7 /
// 15.9 us at M = 1 / 4 / 8 against 16.4 / 16.8 / 17.1 for (8, 2)), (6, 4) up
// to 16 (18.2 us at M = 16; 8 warps of 4 pairs spill, one pipelined pair
// measured 23.7), (4, 4) up to 32 (23.1 / 24.0 us at M = 24 / 32 against
// 27.1 / 27.4 for the tcgen05 GEMV; 6 warps spill there).
template <typename T, int NT, int EPI>
int launch_nt(const GemvMmaParams& p, const kf_gemm_config& cfg, cudaStream_t stream) {
  const int s = cfg.block_m != 0 ? cfg.block_m : (NT == 1 ? 8 : NT == 2 ? 6 : 4);
  const int u = cfg.stages != 0 ? cfg.stages : (NT == 1 ? 1 : 4);
  if (s == 8 && u == 1) return launch_shape<T, NT, 8, 1, EPI>(p, stream);
  if (s == 4 && u == 4) return launch_shape<T, NT, 4, 4, EPI>(p, stream);
  if (s == 4 && u == 2) return launch_shape<T, NT, 4, 2, EPI>(p, stream);
  if (s == 4 && u == 8) return launch_shape<T, NT, 4, 8, EPI>(p, stream);
  if (s == 6 && u == 2) return launch_shape<T, NT, 6, 2, EPI>(p, stream);
  if (s == 6 && u == 4) return launch_shape<T, NT, 6, 4, EPI>(p, stream);
  if (s == 8 && u == 2) return launch_shape<T, NT, 8, 2, EPI>(p, stream);
  if (s == 8 && u == 4) return launch_shape<T, NT, 8, 4, EPI>(p, stream);
  return set_error(KF_ERR_INVALID_CONFIG, "tile GEMV: no compiled shape with " + std::to_string(s) +
                                              " warps per tile and " + std::to_string(u) +
                                              " vector pairs in flight");
}

template <typename T, int EPI>
int launch_epi(const GemvMmaParams& p, const kf_gemm_config& cfg, cudaStream_t stream) {
  if (p.M <= 8) return launch_nt<T, 1, EPI>(p, cfg, stream);
  if (p.M <= 16) return launch_nt<T, 2, EPI>(p, cfg, stream);
  return launch_nt<T, 4, EPI>(p, cfg, stream);
}

template <typename T>
int launch_typed(const GemvMmaParams& p, const kf_gemm_config& cfg, int epilogue, cudaStream_t stream) {
  switch (epilogue) {
    case KF_EPI_NONE: return launch_epi<T, KF_EPI_NONE>(p, cfg, stream);
    case KF_EPI_BIAS: return launch_epi<T, KF_EPI_BIAS>(p, cfg, stream);
    case KF_EPI_BIAS_GELU_TANH: return launch_epi<T, KF_EPI_BIAS_GELU_TANH>(p, cfg, stream);
    case KF_EPI_BIAS_GELU_ERF: return launch_epi<T, KF_EPI_BIAS_GELU_ERF>(p, cfg, stream);
  }
  return set_error(KF_ERR_INVALID_ARGUMENT, "unknown epilogue code");
}

}  // namespace

bool gemv_mma_supported(int dtype, const void* x, int64_t sx_m, int64_t sx_k, const void* w, int64_t sw_n,
                        int64_t sw_k, int64_t M, int64_t N, int64_t K, std::string* why) {
  auto no = [&](const char* msg) {
    if (why) *why = msg;
    return false;
  };
  if (dtype != KF_FP16 && dtype != KF_BF16) return no("the tile GEMV takes fp16 or bf16");
  if (M < 1 || M > GEMV_MMA_MAX_M) return no("the tile GEMV takes 1..32 rows of x");
  if (N > INT32_MAX || K > INT32_MAX) return no("dimensions above 2^31");
  if (K % 8 != 0) return no("K must be a multiple of 8 (whole 16-byte vectors)");
  if (sw_k != 1 || sx_k != 1) return no("weight and x rows must be K-contiguous");
  if ((reinterpret_cast<uintptr_t>(w) & 15u) != 0 || ((sw_n * 2) & 15) != 0)
    return no("weight rows must start on 16-byte boundaries");
  if ((reinterpret_cast<uintptr_t>(x) & 15u) != 0 || (M > 1 && ((sx_m * 2) & 15) != 0))
    return no("x rows must start on 16-byte boundaries");
  return true;
}

int launch_gemv_mma(int dtype, const void* x, int64_t sx_m, const void* w, int64_t sw_n, void* y,
                    int64_t sy_m, int64_t sy_n, int64_t M, int64_t N, int64_t K,
                    const kf_gemm_config& cfg, cudaStream_t stream, int epilogue, const void* bias,
                    void* const* peers, int n_peers, const kf_peer_sync* sync, int* status) {
  if (epilogue != KF_EPI_NONE && bias == nullptr)
    return set_error(KF_ERR_INVALID_ARGUMENT, "epilogue needs a bias pointer");
  if (n_peers < 0 || n_peers > KF_MAX_PEERS || (n_peers > 0 && peers == nullptr))
    return set_error(KF_ERR_INVALID_ARGUMENT, "tile GEMV: bad peer list");
  GemvMmaParams p{};
  p.x = x;
  p.sx_m = sx_m;
  p.w = w;
  p.sw_n = sw_n;
  p.y = y;
  p.sy_m = sy_m;
  p.sy_n = sy_n;
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.bias = bias;
  p.ks = cfg.cluster_m > 0 ? cfg.cluster_m : default_tile_split((N + 15) / 16, static_cast<int>(M));
  if (p.ks != 1 && p.ks != 2 && p.ks != 4 && p.ks != 8)
    return set_error(KF_ERR_INVALID_CONFIG, "tile GEMV: CLUSTER_M (CTAs per weight tile) must be 1, 2, 4 or 8");
  p.n_peers = n_peers;
  for (int j = 0; j < n_peers; ++j) {
    if (peers[j] == nullptr) return set_error(KF_ERR_INVALID_ARGUMENT, "null peer output pointer");
    p.peers[j] = peers[j];
  }
  if (sync != nullptr) {
    if (sync->arrivals == nullptr || sync->epoch_counter == nullptr || sync->local_signals == nullptr ||
        sync->peer_signals == nullptr)
      return set_error(KF_ERR_INVALID_ARGUMENT, "peer sync: null arrival, epoch or signal pointer");
    if (sync->world < 2 || sync->world > KF_MAX_PEERS + 1 || sync->rank < 0 || sync->rank >= sync->world)
      return set_error(KF_ERR_INVALID_ARGUMENT, "peer sync: rank / world out of range");
    if (sync->timeout_us <= 0 || sync->timeout_us > 60000000)
      return set_error(KF_ERR_INVALID_ARGUMENT, "peer sync: timeout_us must be in (0, 6e7]");
    const int rc = fill_peer_signals(sync->local_signals, sync->peer_signals, sync->rank, sync->world,
                                     sync->timeout_us, &p.sig);
    if (rc != KF_OK) return rc;
    p.sync = 1;
    p.arrivals = sync->arrivals;
    p.epoch_counter = sync->epoch_counter;
    p.storing_ctas = static_cast<unsigned int>((N + 15) / 16);
    p.status = status;
  }
  if (N == 0 || M == 0) return KF_OK;
  if (dtype == KF_BF16) return launch_typed<__nv_bfloat16>(p, cfg, epilogue, stream);
  return launch_typed<__half>(p, cfg, epilogue, stream);
}

}  // namespace kf
