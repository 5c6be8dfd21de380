// Streamed tile GEMV: y[m, n] = epi(sum_k x[m, k] w[n, k]) for M <= 16 and a
// weight whose rows are K-contiguous (nn.Linear's [N, K]), fp16/bf16.
//
// The weight is read once, so the kernel is an HBM stream; what limits the
// register-fed tile GEMV (gemv_mma.cu) is how many bytes its warps can keep
// in flight, since each in-flight 16-byte vector holds four registers until it
// lands. Here the bytes in flight live in shared memory instead: one
// persistent CTA per SM keeps a ring of stages (16 weight rows x CH elements,
// 32 KB at CH = 1024) filled by a producer warp with TMA tile loads of 16 rows
// x 256 elements (8 KB each; one thread issues them). Copies of one row's
// 1-2 KB each measured 2.7 / 4.6 TB/s on B200 at CH = 512 / 1024, whatever the
// ring depth: the copy count, not the bytes, set the rate. Out-of-range rows
// (n >= N) and columns (k >= K) arrive as zeros.
//
// Work order: a CTA owns a contiguous run of 16-row tiles (balanced to one
// tile) and walks it in groups of TPG tiles, chunk-major inside a group: for
// each CH-element K chunk, the TPG tiles' stages in turn. Before a chunk's
// weight stages the producer also copies the chunk of x ([16 rows][CH], zeros
// past M and K) into a two-slot x ring; every lane reads its x fragment from
// there once per chunk and it feeds all TPG tiles, so x is read once per group
// and never waited on from global memory (at 16 x 11008 x 4096 loads of x
// from L1/L2 in the consumers measured 19.1-21.1 us alone and 19.2 with
// overlap; the x ring 20.0 and 18.2). Each tile keeps its
// accumulators in registers until the group ends. Then the warps' partial tiles meet in
// shared memory, are summed in warp order (deterministic) and rounded once
// into y after the epilogue (bias, GELU). Consumer warp w reads vectors
// 16w .. 16w + 15 of each row of a stage (its K slice) as mma.sync A
// fragments; the K order inside an MMA is free as long as A and x agree.
//
// With overlap (kf_gemm_config.overlap) the grid is launched as a
// programmatic dependent of the kernel before it on the stream: it may start
// as that kernel's CTAs leave their SMs, its producer issues the first ring of
// weight stages at once (the caller promises the earlier kernel does not write
// the weight) and waits for the earlier grid to complete before it copies any
// x; the consumers wait for it too before they write y. Each CTA lets the
// next such launch start early in turn. Back to
// back, a launch's weight stream fills the SMs its predecessor's last tiles
// leave idle.
//
// Every wait is bounded (KF_WAIT_LIMIT_NS). A failed wait raises the CTA's
// abort flag; the consumer warps run their loops to the end without waiting
// or storing (so every named barrier is met), the producer stops issuing, and
// its thread waits, again bounded, for the copies still in flight before the
// CTA exits, so no copy lands in released shared memory.
//
// Same contract as the reference's matmul at decode shapes
// (kernelforge/kernels/matmul.py:132-155, M in {1, 4, 16}): fp32
// accumulation and one output rounding.
#include <cudaTypedefs.h>

#include <mutex>

#include "kf_common.cuh"
#include "kf_internal.h"

namespace kf {
namespace {

constexpr int ST_WARPS = 8;  // consumer warps; one more warp fills the ring
constexpr int ST_THREADS = 32 * (ST_WARPS + 1);
constexpr int ST_MAX_STAGES = 12;
constexpr int ST_EPI_BAR = 1;  // named barrier of the consumer warps

constexpr int ST_BOX_K = 256;  // elements per row of one TMA box (16 rows x 512 bytes)
constexpr int ST_X_SLOTS = 2;  // chunks of x in flight (each [16 rows][CH], one stage's size)

// A stage: CH / 256 boxes of [16 rows][256 elements], dense.
template <int CH>
struct StageShape {
  static constexpr int boxes = CH / ST_BOX_K;
  static constexpr int bytes = 16 * CH * 2;
  static constexpr int quads = CH / 8 / ST_WARPS / 4;  // vector quads per warp per stage
};

struct GemvStreamParams {
  const void* x;
  long long sx_m;
  const void* w;
  long long sw_n;
  void* y;
  long long sy_m, sy_n;
  const void* bias;
  int M, N, K;
  int tiles;   // ceil(N / 16)
  int chunks;  // ceil(K / CH)
  int stages;  // ring depth
  int overlap;  // launched as a programmatic dependent of the previous kernel
  int* status;
};

// Tiles per group: their accumulators stay in registers for a whole group.
template <int NT>
struct TilesPerGroup {
  static constexpr int value = NT == 1 ? 8 : 6;
};

__device__ __forceinline__ void consumer_bar() {
  asm volatile("bar.sync %0, %1;" ::"n"(ST_EPI_BAR), "n"(32 * ST_WARPS) : "memory");
}
__device__ __forceinline__ bool consumer_bar_and(bool pred) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(out)
      : "r"(static_cast<uint32_t>(pred)), "n"(ST_EPI_BAR), "n"(32 * ST_WARPS)
      : "memory");
  return out != 0;
}

template <typename T, int NT, int CH, int EPI, bool OVERLAP>
__global__ void __launch_bounds__(ST_THREADS, 1)
    gemv_stream_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                       const GemvStreamParams p) {
  constexpr int TPG = TilesPerGroup<NT>::value;
  constexpr int STAGE = StageShape<CH>::bytes;
  constexpr int QUADS = StageShape<CH>::quads;
  constexpr int BOX_BYTES = 16 * ST_BOX_K * 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  uint8_t* xring = ring + static_cast<size_t>(p.stages) * STAGE;  // ST_X_SLOTS chunks of x, same shape
  float4* part = reinterpret_cast<float4*>(xring + ST_X_SLOTS * STAGE);
  uint64_t* full = reinterpret_cast<uint64_t*>(part + ST_WARPS * 32 * NT);
  uint64_t* empty = full + p.stages;
  uint64_t* xfull = empty + p.stages;
  uint64_t* xempty = xfull + ST_X_SLOTS;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(xempty + ST_X_SLOTS);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long grid = gridDim.x;
  const int t_begin = static_cast<int>(static_cast<long long>(p.tiles) * blockIdx.x / grid);
  const int t_end = static_cast<int>(static_cast<long long>(p.tiles) * (blockIdx.x + 1) / grid);

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(smem_u32(full + s), 1);
      mbar_init(smem_u32(empty + s), ST_WARPS);
    }
    for (int s = 0; s < ST_X_SLOTS; ++s) {
      mbar_init(smem_u32(xfull + s), 1);
      mbar_init(smem_u32(xempty + s), ST_WARPS);
    }
    *abort_flag = 0;
    mbar_init_fence();
  }
  __syncthreads();
  // The next launch may be scheduled as this grid's CTAs finish; it waits for
  // this grid's completion before it reads x or writes y.
  if (OVERLAP) griddep_launch_dependents();

  if (warp == ST_WARPS) {
    // ---- producer: one thread walks the consumers' order (groups of TPG
    // tiles, chunk-major inside a group): before a chunk's weight stages, the
    // chunk of x ([16 rows][CH], rows past M are zeros) into the x ring; each
    // stage as CH / 256 box loads.
    if (lane != 0) return;
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_x);
    int slot = 0, xslot = 0;
    uint32_t phase = 0, xphase = 0;
    long long issued = 0, xissued = 0;
    bool ok = true;
    auto issue_w = [&](int tile, int c) {
      if (issued >= p.stages) {  // the slot's previous unit has been read by every consumer warp
        ok = mbar_wait(smem_u32(empty + slot), phase ^ 1u, abort_flag, p.status, SITE_TMA_EMPTY);
        if (!ok) return;
      }
      const uint32_t bar = smem_u32(full + slot);
      const uint32_t dst = smem_u32(ring + static_cast<size_t>(slot) * STAGE);
      mbar_arrive_expect_tx(bar, STAGE);
#pragma unroll
      for (int b = 0; b < StageShape<CH>::boxes; ++b)
        tma_load_2d(dst + b * BOX_BYTES, &tm_w, bar, c * CH + b * ST_BOX_K, tile * 16);
      ++issued;
      if (++slot == p.stages) {
        slot = 0;
        phase ^= 1u;
      }
    };
    // With overlap the first ring of weight stages goes out before the
    // earlier grid has finished (it does not write the weight); x only after.
    long long prefetched = 0;
    if (OVERLAP) {
      for (int tg0 = t_begin; tg0 < t_end && prefetched < p.stages; tg0 += TPG) {
        const int in_group = min(TPG, t_end - tg0);
        for (int c = 0; c < p.chunks && prefetched < p.stages; ++c)
          for (int j = 0; j < in_group && prefetched < p.stages; ++j, ++prefetched) issue_w(tg0 + j, c);
      }
      griddep_wait();
    }
    long long u = 0;
    for (int tg0 = t_begin; tg0 < t_end && ok; tg0 += TPG) {
      const int in_group = min(TPG, t_end - tg0);
      for (int c = 0; c < p.chunks && ok; ++c) {
        if (xissued >= ST_X_SLOTS) {  // every consumer warp has read the slot's previous chunk
          ok = mbar_wait(smem_u32(xempty + xslot), xphase ^ 1u, abort_flag, p.status, SITE_TMA_EMPTY);
          if (!ok) break;
        }
        const uint32_t xbar = smem_u32(xfull + xslot);
        const uint32_t xdst = smem_u32(xring + static_cast<size_t>(xslot) * STAGE);
        mbar_arrive_expect_tx(xbar, STAGE);
#pragma unroll
        for (int b = 0; b < StageShape<CH>::boxes; ++b)
          tma_load_2d(xdst + b * BOX_BYTES, &tm_x, xbar, c * CH + b * ST_BOX_K, 0);
        ++xissued;
        if (++xslot == ST_X_SLOTS) {
          xslot = 0;
          xphase ^= 1u;
        }
        for (int j = 0; j < in_group && ok; ++j, ++u)
          if (u >= prefetched) issue_w(tg0 + j, c);
      }
    }
    // Let every copy land before the CTA can leave: the last units of both
    // rings (all consumed on the normal path, so these waits return at once).
    const long long last = issued < p.stages ? issued : p.stages;
    for (long long v = 0; v < last; ++v) {
      if (slot == 0) {
        slot = p.stages;
        phase ^= 1u;
      }
      --slot;
      mbar_wait(smem_u32(full + slot), phase, nullptr, p.status, SITE_DRAIN, 100000000ull);
    }
    const long long xlast = xissued < ST_X_SLOTS ? xissued : ST_X_SLOTS;
    for (long long v = 0; v < xlast; ++v) {
      if (xslot == 0) {
        xslot = ST_X_SLOTS;
        xphase ^= 1u;
      }
      --xslot;
      mbar_wait(smem_u32(xfull + xslot), xphase, nullptr, p.status, SITE_DRAIN, 100000000ull);
    }
    return;
  }

  // ---- consumers
  const int g = lane >> 2, t = lane & 3;
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
  T* y = static_cast<T*>(p.y);
  const T* bias = static_cast<const T*>(p.bias);
  // y may be the earlier grid's input (x arrives only after it completed,
  // through the producer's wait; this keeps the stores ordered on their own).
  if (OVERLAP) griddep_wait();
  int slot = 0, xslot = 0;
  uint32_t phase = 0, xphase = 0;
  bool ok = true;  // every wait so far succeeded (warp-uniform)
  for (int tg0 = t_begin; tg0 < t_end; tg0 += TPG) {
    const int in_group = min(TPG, t_end - tg0);
    float acc[TPG][NT][4];
#pragma unroll
    for (int j = 0; j < TPG; ++j)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[j][nt][i] = 0.0f;

    for (int c = 0; c < p.chunks; ++c) {
      // This lane's x fragment for the chunk (vectors 4q + t of its warp's K
      // slice, x rows g and g + 8), shared by the group's tiles; the x slot
      // is released as soon as every warp holds its fragment.
      uint4 xv[QUADS][NT];
      {
        bool got = ok && mbar_wait(smem_u32(xfull + xslot), xphase, abort_flag, p.status, SITE_MMA_FULL);
        ok = __all_sync(0xffffffffu, got);
        const uint8_t* xp = xring + static_cast<size_t>(xslot) * STAGE;
#pragma unroll
        for (int q = 0; q < QUADS; ++q) {
          const int v = warp * (4 * QUADS) + 4 * q + t;
          const uint8_t* vp = xp + (v >> 5) * BOX_BYTES + (v & 31) * 16;
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
            xv[q][nt] = ok ? *reinterpret_cast<const uint4*>(vp + (g + 8 * nt) * (ST_BOX_K * 2)) : zero;
        }
        __syncwarp();
        if (ok && lane == 0) mbar_arrive(smem_u32(xempty + xslot));
        if (++xslot == ST_X_SLOTS) {
          xslot = 0;
          xphase ^= 1u;
        }
      }
#pragma unroll
      for (int j = 0; j < TPG; ++j) {
        if (j < in_group) {
          // After a failed wait the loops still run to the end (no wait, no
          // store), so every consumer warp reaches the same named barriers.
          bool got = ok && mbar_wait(smem_u32(full + slot), phase, abort_flag, p.status, SITE_MMA_FULL);
          ok = __all_sync(0xffffffffu, got);
          const uint8_t* sp = ring + static_cast<size_t>(slot) * STAGE;
          uint4 va[QUADS], vb[QUADS];
#pragma unroll
          for (int q = 0; q < QUADS; ++q) {
            // vector v of the chunk: box v / 32, vector v % 32 of its rows
            // (beyond K the box holds zeros)
            const int v = warp * (4 * QUADS) + 4 * q + t;
            const uint8_t* vp = sp + (v >> 5) * BOX_BYTES + (v & 31) * 16;
            va[q] = ok ? *reinterpret_cast<const uint4*>(vp + g * (ST_BOX_K * 2)) : zero;
            vb[q] = ok ? *reinterpret_cast<const uint4*>(vp + (g + 8) * (ST_BOX_K * 2)) : zero;
          }
          __syncwarp();
          if (ok && lane == 0) mbar_arrive(smem_u32(empty + slot));
          if (++slot == p.stages) {
            slot = 0;
            phase ^= 1u;
          }
#pragma unroll
          for (int q = 0; q < QUADS; ++q)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              // vector elements 0-3 then 4-7: logical k {2t, 2t+1, 2t+8, 2t+9}
              mma16816<T>(acc[j][nt], va[q].x, vb[q].x, va[q].y, vb[q].y, xv[q][nt].x, xv[q][nt].y);
              mma16816<T>(acc[j][nt], va[q].z, vb[q].z, va[q].w, vb[q].w, xv[q][nt].z, xv[q][nt].w);
            }
        }
      }
    }

    // The group's tiles: the warps' partial sums meet in shared memory.
    // D fragment: acc[j][nt][0..1] = weight row g, x rows 8nt+2t, +1;
    // [2..3] = weight row g+8.
    const bool all_ok = consumer_bar_and(ok);
#pragma unroll
    for (int j = 0; j < TPG; ++j) {
      if (j < in_group) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
          part[(warp * 32 + lane) * NT + nt] = make_float4(acc[j][nt][0], acc[j][nt][1], acc[j][nt][2], acc[j][nt][3]);
        consumer_bar();
        const int e = threadIdx.x;  // one output value per consumer thread
        if (all_ok && e < 32 * NT * 4) {
          const int ln = e / (NT * 4), nt = (e >> 2) % NT, i = e & 3;
          float s = 0.0f;
#pragma unroll
          for (int w = 0; w < ST_WARPS; ++w) {
            const float* pv = reinterpret_cast<const float*>(&part[(w * 32 + ln) * NT + nt]);
            s += pv[i];
          }
          const int m = 8 * nt + 2 * (ln & 3) + (i & 1);
          const int n = (tg0 + j) * 16 + (ln >> 2) + (i >> 1) * 8;
          if (m < p.M && n < p.N) {
            const float b = EPI != KF_EPI_NONE ? to_f32(bias[n]) : 0.0f;
            y[m * p.sy_m + static_cast<long long>(n) * p.sy_n] = from_f32<T>(apply_epilogue<EPI>(s, b));
          }
        }
        consumer_bar();  // part is rewritten by the next tile
      }
    }
  }
}

// The weight's and x's tensor maps.
struct StreamMaps {
  CUtensorMap w, x;
};

template <typename T, int NT, int CH, int EPI>
int launch_typed(const StreamMaps& maps, const GemvStreamParams& p, size_t smem, int grid, cudaStream_t stream) {
  void* fn = p.overlap ? reinterpret_cast<void*>(gemv_stream_kernel<T, NT, CH, EPI, true>)
                       : reinterpret_cast<void*>(gemv_stream_kernel<T, NT, CH, EPI, false>);
  // The attribute only ever grows: set it once per kernel (and device).
  static thread_local int set_device[2] = {-1, -1};
  static thread_local size_t set_bytes[2] = {0, 0};
  const int o = p.overlap ? 1 : 0;
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return cuda_error(err, "cudaGetDevice");
  if (device != set_device[o] || smem > set_bytes[o]) {
    err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (err != cudaSuccess) return cuda_error(err, "cudaFuncSetAttribute(gemv stream)");
    set_device[o] = device;
    set_bytes[o] = smem;
  }
  CUtensorMap mw = maps.w, mx = maps.x;
  GemvStreamParams q = p;
  void* args[] = {&mw, &mx, &q};
  cudaLaunchConfig_t lc{};
  lc.gridDim = dim3(static_cast<unsigned>(grid));
  lc.blockDim = dim3(ST_THREADS);
  lc.dynamicSmemBytes = smem;
  lc.stream = stream;
  cudaLaunchAttribute attr[1];
  if (p.overlap) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
  }
  err = cudaLaunchKernelExC(&lc, fn, args);
  if (err != cudaSuccess) return cuda_error(err, "launch(gemv_stream_kernel)");
  return KF_OK;
}

template <typename T, int NT, int CH>
int launch_epi(const StreamMaps& tm, const GemvStreamParams& p, int epilogue, size_t smem, int grid,
               cudaStream_t stream) {
  switch (epilogue) {
    case KF_EPI_NONE: return launch_typed<T, NT, CH, KF_EPI_NONE>(tm, p, smem, grid, stream);
    case KF_EPI_BIAS: return launch_typed<T, NT, CH, KF_EPI_BIAS>(tm, p, smem, grid, stream);
    case KF_EPI_BIAS_GELU_TANH: return launch_typed<T, NT, CH, KF_EPI_BIAS_GELU_TANH>(tm, p, smem, grid, stream);
    case KF_EPI_BIAS_GELU_ERF: return launch_typed<T, NT, CH, KF_EPI_BIAS_GELU_ERF>(tm, p, smem, grid, stream);
  }
  return set_error(KF_ERR_INVALID_ARGUMENT, "unknown epilogue code");
}

template <typename T, int CH>
int launch_nt(const StreamMaps& tm, const GemvStreamParams& p, int nt, int epilogue, size_t smem, int grid,
              cudaStream_t stream) {
  return nt == 1 ? launch_epi<T, 1, CH>(tm, p, epilogue, smem, grid, stream)
                 : launch_epi<T, 2, CH>(tm, p, epilogue, smem, grid, stream);
}

// A K-contiguous operand (the weight [N][K], or x [M][K]) as a 2-D tensor
// map, boxes of 16 rows x 256 elements, no swizzle, zeros outside the tensor.
int encode_rows_map(CUtensorMap* map, int dtype, const void* w, int64_t N, int64_t K, int64_t sw_n) {
  static PFN_cuTensorMapEncodeTiled_v12000 enc = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* sym = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &sym, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      enc = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(sym);
  });
  if (enc == nullptr) return set_error(KF_ERR_LAUNCH, "cuTensorMapEncodeTiled unavailable");
  const int64_t row_bytes = N > 1 ? sw_n * 2 : ((K * 2 + 15) / 16) * 16;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(N)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
  cuuint32_t box[2] = {ST_BOX_K, 16};
  cuuint32_t elem_strides[2] = {1, 1};
  const CUtensorMapDataType t = dtype == KF_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const CUresult r = enc(map, t, 2, const_cast<void*>(w), dims, strides, box, elem_strides,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(KF_ERR_UNALIGNED, "streamed tile GEMV: cuTensorMapEncodeTiled rejected an operand (error " +
                                           std::to_string(r) + ")");
  return KF_OK;
}

}  // namespace

bool gemv_stream_supported(int dtype, const void* x, int64_t sx_m, int64_t sx_k, const void* w, int64_t sw_n,
                           int64_t sw_k, int64_t M, int64_t N, int64_t K, std::string* why) {
  if (M > GEMV_STREAM_MAX_M) {
    if (why) *why = "the streamed tile GEMV takes 1..16 rows of x";
    return false;
  }
  // Same operand rules as the register-fed tile kernel: 16-bit, K % 8 == 0,
  // K-contiguous rows on 16-byte boundaries (each row chunk is one bulk copy).
  return gemv_mma_supported(dtype, x, sx_m, sx_k, w, sw_n, sw_k, M, N, K, why);
}

int launch_gemv_stream(int dtype, const void* x, int64_t sx_m, const void* w, int64_t sw_n, void* y,
                       int64_t sy_m, int64_t sy_n, int64_t M, int64_t N, int64_t K, const kf_gemm_config& cfg,
                       const DeviceInfo& dev, cudaStream_t stream, int epilogue, const void* bias) {
  if (epilogue != KF_EPI_NONE && bias == nullptr)
    return set_error(KF_ERR_INVALID_ARGUMENT, "epilogue needs a bias pointer");
  if (M < 1 || M > GEMV_STREAM_MAX_M) return set_error(KF_ERR_UNSUPPORTED, "streamed tile GEMV: 1..16 rows of x");
  // block_k: weight elements per row per stage (one bulk copy each).
  const int ch = cfg.block_k != 0 ? cfg.block_k : GEMV_STREAM_DEFAULT_CHUNK;
  if (ch != 512 && ch != 1024)
    return set_error(KF_ERR_INVALID_CONFIG, "streamed tile GEMV: BLOCK_K (chunk) must be 512 or 1024");
  if (N == 0) return KF_OK;
  GemvStreamParams p{};
  p.x = x;
  p.sx_m = sx_m;
  p.w = w;
  p.sw_n = sw_n;
  p.y = y;
  p.sy_m = sy_m;
  p.sy_n = sy_n;
  p.bias = bias;
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.tiles = static_cast<int>((N + 15) / 16);
  p.chunks = static_cast<int>((K + ch - 1) / ch);
  p.status = dev.status;
  p.overlap = cfg.overlap != 0 ? 1 : 0;
  const int nt = M <= 8 ? 1 : 2;
  const size_t stage = 16 * static_cast<size_t>(ch) * 2;
  // alignment slack, the x ring and its barriers, the warps' partial tiles, the abort flag
  const size_t fixed = 128 + ST_X_SLOTS * (stage + 16) + static_cast<size_t>(ST_WARPS) * 32 * nt * sizeof(float4) + 16;
  // Ring depth: config stages if given, else as many as fit (two mbarriers per stage).
  const int fit = static_cast<int>((static_cast<size_t>(dev.max_smem_optin) - fixed) / (stage + 16));
  const int cap = fit < ST_MAX_STAGES ? fit : ST_MAX_STAGES;
  const int stages = cfg.stages != 0 ? cfg.stages : cap;
  if (stages < 2 || stages > cap)
    return set_error(KF_ERR_INVALID_CONFIG, "streamed tile GEMV: stages must be in 2.." + std::to_string(cap));
  p.stages = stages;
  const size_t smem = fixed + static_cast<size_t>(stages) * (stage + 16);
  // One CTA per SM (num_ctas overrides), never more CTAs than tiles.
  int grid = cfg.num_ctas > 0 ? cfg.num_ctas : dev.sm_count;
  if (grid > p.tiles) grid = p.tiles;
  StreamMaps tm;
  int rc = encode_rows_map(&tm.w, dtype, w, N, K, sw_n);
  if (rc != KF_OK) return rc;
  rc = encode_rows_map(&tm.x, dtype, x, M, K, sx_m);
  if (rc != KF_OK) return rc;
  if (dtype == KF_BF16)
    return ch == 512 ? launch_nt<__nv_bfloat16, 512>(tm, p, nt, epilogue, smem, grid, stream)
                     : launch_nt<__nv_bfloat16, 1024>(tm, p, nt, epilogue, smem, grid, stream);
  return ch == 512 ? launch_nt<__half, 512>(tm, p, nt, epilogue, smem, grid, stream)
                   : launch_nt<__half, 1024>(tm, p, nt, epilogue, smem, grid, stream);
}

}  // namespace kf
