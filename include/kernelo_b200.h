/*
 * kernelo_b200.h -- C ABI of the B200 (sm_100a) KernelForge hot path.
 *
 * Every entry point takes raw device pointers, int64 sizes and ELEMENT strides,
 * a dtype code, an optional config struct and a cudaStream_t passed as void*.
 * Nothing here allocates or frees device memory, synchronises, or keeps state
 * beyond per-device caches (SM count, the tensor-map encoder) and one device
 * status word per GPU. Kernels are launched asynchronously on `stream`.
 *
 * Each entry point replaces the launch site of one reference wrapper; the
 * citations are file:line in the KernelForge sources (package `kernelforge`):
 *
 *   kf_gemm             kernels/matmul.py:132-155        matmul(a, b, config=)
 *   kf_linear_bias_act  kernels/fused_linear.py:112-157  fused_linear_gelu(x, w, bias, config=)
 *   kf_gemv             kernels/matmul.py:132-155 at M in {1,4,16}
 *                       (the decode-shape GEMM; the reference has no dedicated kernel)
 *   kf_softmax_rows     kernels/softmax.py:70-104        softmax(x, config=)
 *   kf_rmsnorm_rows     kernels/rmsnorm.py:81-127        rmsnorm(x, gamma, eps=, config=)
 *                       and csrc/rmsnorm.cu:19-57        (the hand-written CUDA baseline)
 *   kf_query_gemm_config  tuning/search.py:299-394      shared-memory / feasibility model
 *   kf_gemv_noalloc     as kf_gemv, for callers that cannot hand over a workspace
 *   kf_linear_bias_act_allgather, kf_peer_barrier(_counted), kf_ipc_handle / _open / _close
 *                       the column-sharded fused linear over several GPUs (the
 *                       reference is single-GPU: no counterpart)
 *
 * Status codes are returned by value; kf_last_error() gives the message of the
 * most recent failure on the calling thread.
 */
#ifndef KERNELO_B200_H
#define KERNELO_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KF_ABI_VERSION 1

/* Exported from the shared library (it is built with -fvisibility=hidden). */
#if defined(__GNUC__)
#define KF_API __attribute__((visibility("default")))
#else
#define KF_API
#endif

/* ---- status codes ------------------------------------------------------- */
enum kf_status {
  KF_OK = 0,
  KF_ERR_INVALID_ARGUMENT = 1, /* null pointer, negative size, bad dtype code      */
  KF_ERR_INVALID_CONFIG = 2,   /* config cannot run on this device / these shapes  */
  KF_ERR_UNALIGNED = 3,        /* strides or pointers unusable by the chosen kernel */
  KF_ERR_LAUNCH = 4,           /* the CUDA runtime rejected the launch              */
  KF_ERR_TIMEOUT = 5,          /* a bounded device-side wait gave up (status word)  */
  KF_ERR_UNSUPPORTED = 6,      /* dtype/shape combination has no kernel             */
  KF_ERR_WORKSPACE = 7,        /* workspace missing or too small                    */
  KF_ERR_NO_DEVICE = 8         /* no usable sm_100 device                           */
};

/* ---- dtype codes (kernelforge/dtypes.py:13-17) -------------------------- */
enum kf_dtype { KF_FP16 = 0, KF_BF16 = 1, KF_FP32 = 2 };

/* ---- GEMM epilogues (kernels/fused_linear.py:94-104) -------------------- */
enum kf_epilogue {
  KF_EPI_NONE = 0,           /* C = A.B                                   */
  KF_EPI_BIAS = 1,           /* C = A.B + bias[n]                         */
  KF_EPI_BIAS_GELU_TANH = 2, /* C = gelu_tanh(A.B + bias[n]) (reference)  */
  KF_EPI_BIAS_GELU_ERF = 3   /* C = gelu_erf(A.B + bias[n])  (exact form) */
};

/* ---- GEMM kernels -------------------------------------------------------- */
enum kf_gemm_kernel {
  KF_GEMM_AUTO = 0,    /* library default for the shape                     */
  KF_GEMM_TCGEN05 = 1, /* TMA + tcgen05.mma + TMEM, persistent, fp16/bf16    */
  KF_GEMM_SIMT = 2,    /* CUDA-core FFMA, any strides, fp16/bf16/fp32        */
  KF_GEMM_WARP_ROWS = 3, /* kf_gemv only: a warp per K-contiguous weight row,
                           M <= 4, packed fp32x2 FMA; num_ctas = grid size   */
  KF_GEMM_TILE_ROWS = 4, /* a CTA per 16 K-contiguous weight rows (B's columns),
                           M <= 32, fp16/bf16, K % 8 == 0; the weight registers
                           feed mma.sync.m16n8k16 directly; block_m = warps
                           per tile (K slices), stages = 16-byte vector pairs
                           per lane in flight. kf_gemv, and kf_gemm /
                           kf_linear_bias_act (epilogue included); AUTO picks
                           it for such shapes                               */
  KF_GEMM_COLUMNS = 5,   /* a lane per 16-byte vector of an N-contiguous B's
                           columns (the row-major (K, N) operand), M <= 8,
                           any dtype; K split over CTAs, the last arrival per
                           column strip adds the partials in a fixed order
                           (workspace from kf_gemm_workspace_bytes; without
                           it, one CTA per strip). AUTO picks it for such
                           shapes; epilogue included                        */
  KF_GEMM_TILE_STREAM = 6 /* the 16-row tile GEMV with the weight streamed
                           through shared memory: one persistent CTA per SM
                           keeps a ring of bulk copies (16 rows x 512
                           elements per stage) in flight; M <= 16, the
                           TILE_ROWS operand rules, no workspace; stages =
                           ring depth (2..12), num_ctas = grid size. kf_gemv
                           and kf_gemm / kf_linear_bias_act without peers   */
};

/* Tunable GEMM parameters. Replaces KernelConfig's BLOCK_M/BLOCK_N/BLOCK_K/
 * GROUP_M/num_stages keys (kernels/matmul.py:118-120) with their sm_100a
 * meaning. Zero in any field selects the library default. */
typedef struct kf_gemm_config {
  int32_t kernel;    /* enum kf_gemm_kernel                                         */
  int32_t block_m;   /* tcgen05: 128 (one SM) or 256 (an SM pair, cta_group::2);
                        SIMT: 64 or 128                                              */
  int32_t block_n;   /* tcgen05: multiple of 16 (32 for pairs) in [16,256];
                        SIMT: 64 or 128                                              */
  int32_t block_k;   /* tcgen05: 64 or 128; SIMT: 8 or 16                            */
  int32_t stages;    /* tcgen05 shared-memory ring depth                             */
  int32_t group_m;   /* grouped (L2-aware) raster width, in M tiles                  */
  int32_t stream_k;  /* tcgen05: 0 = library choice, 1 = split K over the persistent
                        grid (stream-K), 2 = whole tiles only, 3 = split tail:
                        whole tiles for the full waves, the last partial wave as
                        half-width tiles (no workspace). A library choice that
                        needs workspace the call did not pass falls back to
                        whole tiles.                                               */
  int32_t swap_ab;   /* tcgen05: 0 = library choice, 1 = compute C^T = B^T.A^T
                        (skinny M), 2 = never swap                                     */
  int32_t cluster_m; /* 1, or 2 with block_m 256 (the SM pair is a 2x1 cluster)      */
  int32_t cluster_n; /* reserved, must be 0 or 1                                     */
  int32_t num_ctas;  /* persistent grid size; 0 = one CTA per SM                     */
  int32_t epi_store; /* all-gather epilogue (kf_linear_bias_act_allgather): 0 = library
                        choice, 1 = stores from the threads (rows staged through
                        shared memory), 2 = TMA tensor stores of the staged blocks    */
  int32_t overlap;   /* decode GEMV (kf_gemv, and kf_gemm / kf_linear_bias_act at
                        M <= 16 without peers): 1 = the weight and bias are not
                        written by the kernel that runs before this call on the
                        stream, so the launch may start as that kernel's CTAs
                        finish (programmatic dependent launch): it streams the
                        weight at once and waits for the earlier kernel to
                        complete before it reads x or writes y. Runs on
                        TILE_STREAM (AUTO picks it where it is faster so);
                        other kernels ignore it.
                        0 = ordinary stream order                                    */
  int32_t reserved[3];
} kf_gemm_config;

/* Row-kernel parameters (softmax / RMSNorm). Replaces BLOCK_SIZE /
 * ROWS_PER_PROGRAM / num_warps (kernels/softmax.py:61-67). */
typedef struct kf_rows_config {
  int32_t num_warps;        /* warps per row: per CTA (register kernel, 1..32) or per
                               row group (streaming kernel, 1..16)                   */
  int32_t rows_per_cta;     /* register kernel: rows one CTA (or cluster) handles     */
  int32_t cluster;          /* register kernel: CTAs sharing one row through DSMEM    */
  int32_t kernel;           /* KF_ROWS_AUTO, KF_ROWS_REGISTER, KF_ROWS_STREAM or
                               KF_ROWS_WARP                                         */
  int32_t row_groups;       /* streaming kernel: row groups per CTA (0 = 16 / num_warps) */
  int32_t stages;           /* streaming kernel: shared-memory row slots per row group
                               (0 = as many as fit, at most 8)                        */
  int32_t reserved[2];
} kf_rows_config;

/* Peers an all-gathering call can write to: an 8-GPU node. */
#define KF_MAX_PEERS 7

/* Row kernels. REGISTER: one row per CTA (or per cluster of up to 8 CTAs for
 * wide rows), loaded straight into registers. STREAM: persistent CTAs (one or
 * two per SM) of row groups; each group keeps its next rows in flight as bulk
 * copies into shared-memory slots while it reduces and writes earlier ones.
 * WARP: persistent CTAs of 8 warps, a warp per row, the next row loaded into
 * registers while the current one is reduced; rows of up to 4 KB that start on
 * the 16-byte grid (the default for such softmax rows up to 2 KB, RMSNorm rows
 * up to 4 KB). */
enum kf_rows_kernel { KF_ROWS_AUTO = 0, KF_ROWS_REGISTER = 1, KF_ROWS_STREAM = 2, KF_ROWS_WARP = 3 };

/* ---- library information -------------------------------------------------- */
KF_API int32_t kf_abi_version(void);
KF_API const char* kf_version(void);
/* Message of the last failing call on this thread ("" if none). */
KF_API const char* kf_last_error(void);
/* Number of SMs of `device` (cached), or a negative status. */
KF_API int32_t kf_sm_count(int32_t device);

/* Reads and clears the device status word of `device` (synchronises that device).
 * *out receives KF_OK or KF_ERR_TIMEOUT with the kernel site in the high bits. */
KF_API int32_t kf_device_status(int32_t device, int32_t* out);

/* ---- GEMM: C[M,N] = A[M,K] . B[K,N] --------------------------------------- *
 * Strides are in elements: A(m,k) = a[m*sa_m + k*sa_k], B(k,n) = b[k*sb_k + n*sb_n],
 * C(m,n) = c[m*sc_m + n*sc_n]. Accumulation is fp32; C has the operand dtype.
 * fp32 beyond 64 x 64 and 2^27 multiply-adds (or with KF_GEMM_TCGEN05) runs as
 * 3xTF32 on tensor cores: A and B are split into TF32 parts in the workspace
 * and a kind::tf32 GEMM sums a_small b_big + a_big b_small + a_big b_big, which
 * holds the fp32 gate (1e-5); smaller fp32 problems, and calls given too
 * little workspace, run IEEE FMA on CUDA cores.
 * `workspace` holds stream-K state and any operand copies;
 * kf_gemm_workspace_bytes_for() gives its size (256-byte aligned). Layout:
 * 64 KiB of per-tile arrival counters, then fp32 partial tiles, then copies.
 * The counters must be zero before the first use; every call leaves them zero
 * again, so one zeroed buffer can serve any sequence of calls on one stream
 * (calls that overlap on the GPU race). */
KF_API int32_t kf_gemm(int32_t dtype, const void* a, int64_t sa_m, int64_t sa_k, const void* b,
                int64_t sb_k, int64_t sb_n, void* c, int64_t sc_m, int64_t sc_n, int64_t M,
                int64_t N, int64_t K, const kf_gemm_config* cfg, void* workspace,
                int64_t workspace_bytes, void* stream);

/* Y = act(X . W + bias). W(k,n) = w[k*sw_k + n*sw_n]: both the reference's (K,N)
 * layout and nn.Linear's [N,K] layout (sw_k = 1) are accepted without copies. */
KF_API int32_t kf_linear_bias_act(int32_t dtype, const void* x, int64_t sx_m, int64_t sx_k,
                           const void* w, int64_t sw_k, int64_t sw_n, const void* bias,
                           void* y, int64_t sy_m, int64_t sy_n, int64_t M, int64_t N, int64_t K,
                           int32_t epilogue, const kf_gemm_config* cfg, void* workspace,
                           int64_t workspace_bytes, void* stream);

/* Decode-shape GEMM Y[M,N] = X[M,K] . W^T for small M (1..256) with W stored
 * [N,K] (sw_n = row stride, sw_k = 1) or [K,N] (sw_k = row stride, sw_n = 1).
 * Memory-bound. The default config picks by layout: fp16/bf16 with
 * K-contiguous W and x rows and M <= 32 run the 16-row tile kernel (W streamed
 * by warps into mma.sync fragments, no workspace), or at 9..16 rows with
 * K >= 8192 or at least eight 16-row tiles per SM, and with cfg->overlap
 * beyond 8 rows, for K >= 8192 or below four tiles per SM, the streamed tile
 * kernel (KF_GEMM_TILE_STREAM, no workspace); fp32 at M <= 2 the
 * warp-per-row kernel (no workspace); the rest the tcgen05 GEMV with A and B
 * swapped and K split over all SMs (stream-K), which uses
 * kf_gemv_workspace_bytes() of workspace when given one and whole tiles
 * otherwise. Operands TMA cannot describe take the CUDA-core GEMM. */
KF_API int32_t kf_gemv(int32_t dtype, const void* x, int64_t sx_m, int64_t sx_k, const void* w,
                int64_t sw_n, int64_t sw_k, void* y, int64_t sy_m, int64_t sy_n, int64_t M,
                int64_t N, int64_t K, const kf_gemm_config* cfg, void* workspace,
                int64_t workspace_bytes, void* stream);

/* kf_gemv for callers that cannot allocate device memory. No counterpart in
 * the reference: it exists for callers such as a plugin inside a host
 * application that owns all device memory and provides neither an allocator
 * nor a workspace, or a latency-critical path that cannot pay for
 * cudaMalloc/cudaFree (which may synchronise the device). Same arguments as
 * kf_gemv minus the config and workspace, and the same kernel choice as
 * kf_gemv's default config: the stream-K scratch is a file-scope device array
 * of KF_NOALLOC_SCRATCH_BYTES inside the library, present on every GPU that
 * loads it until the process exits. Takes M <= KF_NOALLOC_MAX_ROWS and
 * rejects larger M, and any call whose stream-K scratch would not fit the
 * array (x with unit stride along M, for example), with KF_ERR_WORKSPACE
 * before launching anything. Calls no allocating routine. The first call on a
 * device looks the array up (cudaGetSymbolAddress) and should come before any
 * stream capture. Calls on the tile kernel never touch the array; the others
 * clear its counters on `stream`. All calls on a device share the array, so
 * such calls that overlap on the GPU race. */
#define KF_NOALLOC_SCRATCH_BYTES (4 * 1024 * 1024)
#define KF_NOALLOC_MAX_ROWS 16
KF_API int32_t kf_gemv_noalloc(int32_t dtype, const void* x, int64_t sx_m, int64_t sx_k,
                               const void* w, int64_t sw_n, int64_t sw_k, void* y, int64_t sy_m,
                               int64_t sy_n, int64_t M, int64_t N, int64_t K, void* stream);

/* Workspace bytes a kf_gemm / kf_linear_bias_act (resp. kf_gemv) call with
 * these strides, sizes and config needs on `device` (0 when none; negative
 * status on error). Operand pointers are assumed 16-byte aligned and C
 * contiguous. The workspace holds the stream-K counters and partial tiles,
 * the column GEMV's partial sums, the packed copies of fp16/bf16 operands
 * that a TMA tensor map cannot describe (an odd row pitch or K < 8), the
 * TF32-split copies of fp32 operands (2 x 4 bytes per element, K rounded up
 * to 32) and the staged copy of an output whose rows are off the 16-byte
 * grid, these copies after the first 64 KiB. */
KF_API int64_t kf_gemm_workspace_bytes(int32_t device, int32_t dtype, int64_t sa_m, int64_t sa_k,
                                int64_t sb_k, int64_t sb_n, int64_t M, int64_t N, int64_t K,
                                const kf_gemm_config* cfg);
/* kf_gemm_workspace_bytes for these operands and output: an operand whose base
 * is off the 16-byte grid (a view starting at an odd column) is packed too,
 * and an output whose rows are off the 16-byte grid (an odd N) is written to
 * a staged copy first; both are sized for. kf_gemm_workspace_bytes assumes
 * aligned bases and a contiguous C. The ctypes layer behind kernelforge's
 * matmul / fused_linear_gelu wrappers (kernels/matmul.py:132-155,
 * fused_linear.py:112-157) sizes every workspace with it. */
KF_API int64_t kf_gemm_workspace_bytes_for(int32_t device, int32_t dtype, const void* a, int64_t sa_m,
                                           int64_t sa_k, const void* b, int64_t sb_k, int64_t sb_n, void* c,
                                           int64_t sc_m, int64_t sc_n, int64_t M, int64_t N, int64_t K,
                                           const kf_gemm_config* cfg);
KF_API int64_t kf_gemv_workspace_bytes(int32_t device, int32_t dtype, int64_t sx_m, int64_t sx_k,
                                int64_t sw_n, int64_t sw_k, int64_t M, int64_t N, int64_t K,
                                const kf_gemm_config* cfg);

/* Feasibility model used by the tuner's filters (tuning/search.py:299-394).
 * Fills the shared memory (bytes) and TMEM columns a tcgen05 config needs;
 * returns KF_OK or KF_ERR_INVALID_CONFIG. Needs no GPU. */
KF_API int32_t kf_query_gemm_config(int32_t dtype, const kf_gemm_config* cfg, int64_t* smem_bytes,
                             int32_t* tmem_cols);

/* ---- row kernels ----------------------------------------------------------- *
 * y[r, :] = softmax(x[r, :]) over `cols`; fp32 math, output in the input dtype.
 * Row strides in elements; the last dimension must be contiguous. */
KF_API int32_t kf_softmax_rows(int32_t dtype, const void* x, int64_t sx_row, void* y, int64_t sy_row,
                        int64_t rows, int64_t cols, const kf_rows_config* cfg, void* stream);

/* y[r, :] = x[r, :] * rsqrt(mean(x[r, :]^2) + eps) * gamma; fp32 reduction,
 * one rounding at the end (kernels/rmsnorm.py:130-143). */
KF_API int32_t kf_rmsnorm_rows(int32_t dtype, const void* x, int64_t sx_row, const void* gamma,
                        void* y, int64_t sy_row, int64_t rows, int64_t cols, float eps,
                        const kf_rows_config* cfg, void* stream);

/* ---- fused linear + all-gather over NVLink ---------------------------------- *
 * kf_linear_bias_act, and every output tile is also stored into the n_peers
 * buffers y_peers[i]: device pointers (peer-mapped, e.g. symmetric memory) to
 * the element that corresponds to y[0,0] in each peer's copy of Y, which has
 * y's strides. A rank of a column-sharded linear passes its column block of
 * its own Y as y and the same block of every peer's Y as y_peers: when every
 * rank's call has finished and kf_peer_barrier has run, every rank holds all
 * of Y with no collective and no copy. The epilogue ends with a system-scope
 * fence. Runs on the tcgen05 GEMM, or at M <= 32 with a K-contiguous 16-bit
 * weight on the 16-row tile GEMV (the decode-shape layer; epilogue KF_EPI_NONE
 * with a null bias gives the plain sharded GEMV); n_peers <= KF_MAX_PEERS.
 * No reference counterpart: the reference is single-GPU; this replaces the
 * NCCL all_gather of the column-sharded fused linear and decode GEMV. */
KF_API int32_t kf_linear_bias_act_allgather(int32_t dtype, const void* x, int64_t sx_m, int64_t sx_k,
                                            const void* w, int64_t sw_k, int64_t sw_n,
                                            const void* bias, void* y, int64_t sy_m, int64_t sy_n,
                                            int64_t M, int64_t N, int64_t K, int32_t epilogue,
                                            void* const* y_peers, int32_t n_peers,
                                            const kf_gemm_config* cfg, void* workspace,
                                            int64_t workspace_bytes, void* stream);

/* Cross-GPU barrier on the stream: writes `epoch` into slot `rank` of every
 * peer's signal array (release, system scope) and waits -- at most
 * timeout_us microseconds -- until every peer's slot in the local array holds
 * `epoch` (acquire, system scope). local_signals / peer_signals[i] are
 * peer-mapped arrays of `world` uint32 (zero-initialised; epochs increase
 * from 1). A timeout records KF_ERR_TIMEOUT in the device status word (read
 * with kf_device_status) and the kernel returns: it never waits without
 * limit. peer_signals lists the OTHER ranks in rank order. */
KF_API int32_t kf_peer_barrier(uint32_t* local_signals, uint32_t* const* peer_signals,
                               int32_t rank, int32_t world, uint32_t epoch, int32_t timeout_us,
                               void* stream);

/* kf_peer_barrier with the epoch kept on the device: epoch_counter is a
 * uint32 in this rank's memory (zero-initialised, used by nothing else); each
 * barrier takes *epoch_counter + 1 as its epoch and stores it back. Every rank
 * runs the same sequence of barriers, so the counters agree, and the call can
 * be captured once in a CUDA graph and replayed: each replay advances the
 * epoch. Do not mix it with kf_peer_barrier on the same signal arrays. */
KF_API int32_t kf_peer_barrier_counted(uint32_t* local_signals, uint32_t* const* peer_signals,
                                       int32_t rank, int32_t world, uint32_t* epoch_counter,
                                       int32_t timeout_us, void* stream);

/* The bounded cross-GPU barrier that completes an all-gather, as one struct
 * (kf_peer_barrier_counted's arguments plus an arrival word): `arrivals` is a
 * zeroed 4-byte device word of this rank, used and left at zero by the fused
 * form below. */
typedef struct kf_peer_sync {
  uint32_t* local_signals;        /* this rank's signal array [world]            */
  uint32_t* const* peer_signals;  /* the other ranks' arrays, rank order, this
                                     rank skipped                               */
  int32_t rank, world;
  uint32_t* epoch_counter;        /* this rank's epoch word (device)             */
  uint32_t* arrivals;             /* zeroed device word of this rank             */
  int32_t timeout_us;
  int32_t reserved;
} kf_peer_sync;

/* kf_linear_bias_act_allgather followed by kf_peer_barrier_counted, in one
 * launch where the all-gather runs on the 16-row tile GEMV (M <= 32): the
 * last CTA to finish (found by an atomic on `sync->arrivals`) runs the barrier
 * itself, so no second kernel is launched. On the tcgen05 path the barrier
 * kernel follows the GEMM on `stream`. Either way the peers' copies of Y hold
 * every rank's block once this call's work on `stream` is done. */
KF_API int32_t kf_linear_bias_act_allgather_sync(int32_t dtype, const void* x, int64_t sx_m, int64_t sx_k,
                                                 const void* w, int64_t sw_k, int64_t sw_n, const void* bias,
                                                 void* y, int64_t sy_m, int64_t sy_n, int64_t M, int64_t N,
                                                 int64_t K, int32_t epilogue, void* const* y_peers,
                                                 int32_t n_peers, const kf_peer_sync* sync,
                                                 const kf_gemm_config* cfg, void* workspace,
                                                 int64_t workspace_bytes, void* stream);

/* Peer mapping for the all-gather buffers, by CUDA IPC (no multicast object).
 * kf_ipc_handle: the IPC handle (KF_IPC_HANDLE_BYTES bytes) of the allocation
 * holding `ptr`, and ptr's byte offset in it. kf_ipc_open: map a handle from
 * another process on this device; the peer's pointer is *base_out + offset.
 * kf_ipc_close: unmap (pass the base kf_ipc_open returned). */
#define KF_IPC_HANDLE_BYTES 64
KF_API int32_t kf_ipc_handle(const void* ptr, void* handle_out, int64_t* offset_out);
KF_API int32_t kf_ipc_open(const void* handle, void** base_out);
KF_API int32_t kf_ipc_close(void* base);

/* ---- failure-detection self test ------------------------------------------- *
 * Launches one CTA that waits on an mbarrier nothing will ever complete, with
 * a limit of `timeout_us` microseconds, then records KF_ERR_TIMEOUT in the
 * device status word and returns. Exercises the bounded-wait path without
 * hanging or faulting the GPU. */
KF_API int32_t kf_selftest_bounded_wait(int32_t timeout_us, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KERNELO_B200_H */
