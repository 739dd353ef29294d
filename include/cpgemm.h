/*
 * cpgemm.h -- C ABI of the B200 (sm_100a) GEMM that replaces the reference's CuTe-DSL GemmSM90.
 *
 * Reference surface (adelmuursepp/cutedsl_pingpong_gemm) and the entry point that replaces it:
 *
 *   GemmSM90.__init__(tile_shape_mn, epi_tile_mn, cluster_shape_mnk, atom_layout_mn, ab_stage,
 *                     epi_stage, raster_order, reuse_ab, is_persistent, gemm_n_prologue)
 *       gemm_base.py:50-122                      -> cpg_config_validate
 *   cute.compile(gemm, a, b, c, stream)          gemm_base.py:608 (traces GemmSM90.__call__,
 *       gemm_base.py:124-160: layouts, TMA atoms, scheduler params, grid)
 *                                                -> cpg_gemm_create
 *   compiled_gemm(a, b, c, stream)               gemm_base.py:609 (kernel launch :151-160)
 *                                                -> cpg_gemm_run
 *   FastDivmod.create / div / divmod             fast_math.py:56-81
 *                                                -> cpg_fast_divmod_create / cpg_fast_divmod_div
 *   SimpleTileScheduler.Params.create            tile_scheduler.py:50-78
 *                                                -> cpg_sched_params_create
 *   SimpleTileScheduler.get_grid_shape           tile_scheduler.py:110-123 -> cpg_sched_grid_shape
 *   SimpleTileScheduler._map_cta_coords          tile_scheduler.py:125-146
 *                                                -> cpg_sched_cluster_map (host),
 *                                                   cpg_sched_cluster_map_device (device)
 *   get_max_active_clusters(cluster_size)        tile_scheduler.py:20-22 -> cpg_max_active_clusters
 *
 * Conventions: every function returns CPG_OK (0) or a negative CPG_ERR_* code; no exception or
 * abort crosses this boundary.  cpg_strerror() names a code and cpg_last_error_message() gives
 * the detail of the calling thread's last failure.  The caller owns A, B, D (device memory);
 * cpg_gemm_run is stream-ordered and asynchronous, writes D in place and returns without
 * synchronising, like the reference's compiled kernel call.  Matrices are row-major with
 * explicit row strides in elements: A [M,K] (K contiguous), B [N,K] (K contiguous), D [M,N]
 * (N contiguous), i.e. D = A . B^T as in gemm_base.py:587-590.
 */
#ifndef CPGEMM_H_
#define CPGEMM_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CPG_OK 0
#define CPG_ERR_INVALID_CONFIG (-1)  /* a constructor assert of gemm_base.py:72-74, :87, :113, :122 */
#define CPG_ERR_INVALID_SHAPE (-2)   /* negative/oversized extents, strides below the extent */
#define CPG_ERR_ALIGNMENT (-3)       /* TMA needs 16-byte aligned bases and row strides */
#define CPG_ERR_DTYPE (-4)           /* element types other than the supported ones */
#define CPG_ERR_UNSUPPORTED (-5)     /* a valid reference config this build does not implement */
#define CPG_ERR_NO_DEVICE (-6)       /* no sm_100 device, or the device cannot run the kernel */
#define CPG_ERR_CUDA (-7)            /* a CUDA runtime/driver call failed */
#define CPG_ERR_DEVICE_TIMEOUT (-8)  /* a kernel wait ran past its deadline (see status) */
#define CPG_ERR_SMEM (-9)            /* the requested stages do not fit in shared memory */
#define CPG_ERR_NULL (-10)           /* a required pointer argument is NULL */

/* Element types. */
#define CPG_DTYPE_BF16 0
#define CPG_DTYPE_E4M3 1
#define CPG_DTYPE_F32 2

/* FP8 scale modes.  TENSOR: optional per-tensor scales (cpg_epilogue.scale_a / scale_b point to
 * one fp32 each).  BLOCK: scale_a points to A's 1 x 128 scales laid out [ceil(K/128)][M] and
 * scale_b to B's 128 x 128 scales laid out [ceil(N/128)][ceil(K/128)] (both fp32); requires
 * tile_n = 128 or 256 and BF16 output. */
#define CPG_SCALE_TENSOR 0
#define CPG_SCALE_BLOCK 1

/* Raster order of the tile scheduler (tile_scheduler.py:24-27). */
#define CPG_RASTER_ALONG_M 0
#define CPG_RASTER_ALONG_N 1

typedef struct cpg_fast_divmod {
  int32_t divisor;
  uint32_t multiplier;
  uint32_t shift_right;
} cpg_fast_divmod;

/* SimpleTileScheduler.Params (tile_scheduler.py:38-48). */
typedef struct cpg_sched_params {
  int32_t ncluster_m, ncluster_n, ncluster_l;
  int32_t raster_order;
  cpg_fast_divmod dm_clusters_per_problem;
  int32_t num_groups_regular;
  cpg_fast_divmod dm_group_size;
  cpg_fast_divmod dm_group_size_tail;
  cpg_fast_divmod dm_num_clusters_in_group;
  int32_t cluster_m, cluster_n;
  int32_t is_persistent;
} cpg_sched_params;

/* GemmSM90 constructor arguments (gemm_base.py:50-62) plus the scheduler group size, which the
 * reference fixes at 8 (gemm_base.py:65), and the scheduling mode. */
typedef struct cpg_gemm_config {
  int32_t tile_m, tile_n;
  int32_t epi_tile_m, epi_tile_n;
  int32_t cluster_m, cluster_n, cluster_k;
  int32_t atom_m, atom_n;
  int32_t ab_stage, epi_stage;
  int32_t raster_order;
  int32_t reuse_ab, is_persistent, gemm_n_prologue;
  int32_t group_size;
  int32_t dynamic_scheduler; /* 0: the static schedule of tile_scheduler.py (persistent or one
                                tile per cluster); 1: dynamic (cluster launch control): the grid
                                holds one cluster per cluster tile and running clusters take over
                                clusters that have not started, so SMs busy with other work take
                                fewer tiles.  The cluster id -> tile map of the static schedule,
                                except that group_size is lowered until a group's re-read
                                operand panel (AlongN: its B rows over one K range; AlongM: its A
                                rows) is at most 32 MiB; needs reuse_ab = 0 and no Stream-K;
                                ignores is_persistent. */
} cpg_gemm_config;

/* Problem description fixed at create time (the reference fixes dtypes and layouts at compile
 * time and takes M, N, K symbolically; here they are fixed per plan). */
typedef struct cpg_gemm_problem {
  int64_t m, n, k;
  int64_t lda, ldb, ldd; /* row strides in elements */
  int32_t dtype_ab;      /* CPG_DTYPE_BF16 or CPG_DTYPE_E4M3 (A and B share one type) */
  int32_t dtype_d;       /* CPG_DTYPE_BF16, or CPG_DTYPE_F32 for split-K partials */
  int32_t scale_mode;    /* CPG_SCALE_TENSOR, or CPG_SCALE_BLOCK for block-scaled E4M3 */
  int32_t split_k;       /* 0 or 1: none; S > 1: K is cut into S ranges scheduled as the L
                            dimension, and the ranges add their FP32 partial sums into D
                            (dtype_d must be CPG_DTYPE_F32; D is cleared by cpg_gemm_run);
                            CPG_SPLIT_K_STREAM: Stream-K, every resident cluster takes an equal
                            share of all (tile, k-block) pairs; with FP32 D the shares add into
                            D, with BF16 D the last contributor of each tile finishes it from
                            an FP32 workspace the plan owns (no memset, no cast);
                            CPG_SPLIT_K_HYBRID, CPG_SPLIT_K_DECODE (M <= 128): see below.
                            Activations, C and gated need 0/1 */
  int32_t gated;         /* 0, or 1: gated FFN (e.g. SwiGLU).  B holds [W_gate; W_up] as 2N rows
                            of K (ldb its row stride), D is M x N and
                            D[:, n] = act(alpha s_a s_b A . W_gate[n]) * alpha s_a s_b A . W_up[n];
                            needs tile_n 512 (each tile: 256 gate + 256 up accumulator columns),
                            no bias, no C source and no split-K */
  int64_t l;             /* batches: the L mode of the reference's (M, K, L) tensors, which its
                            kernel fixes at one (gemm_base.py:221, tile_scheduler.py:96); 0 or 1:
                            one batch.  Batch b of A, B and D starts batch_stride_* elements
                            after batch b - 1 (multiples of 16 bytes; D's batches must not
                            overlap: batch_stride_d >= m * ldd).  Not with block scales. */
  int64_t batch_stride_a, batch_stride_b, batch_stride_d;
  int32_t grouped;       /* 0, or 1: grouped GEMM (ragged groups, e.g. the experts of an MoE
                            layer).  l is the number of groups G; A is [m, k] with the rows of
                            every group one after the other, B is [G, n, k] (batch_stride_b
                            between groups), D is [m, n]; the group boundaries are given per
                            call to cpg_gemm_run_grouped.  Needs a persistent kernel; no split-K,
                            no block scales, K > 0. */
} cpg_gemm_problem;

#define CPG_SPLIT_K_STREAM (-1)
/* Data-parallel waves + Stream-K tail: the tiles of all full waves but the last are computed
 * whole; the k-blocks of the remaining tiles are shared evenly by the resident clusters, and
 * the last contributor of a split tile finishes it (bias, rounding, store) from an FP32
 * workspace the plan owns.  For problems whose tiles leave the last wave partly idle. */
#define CPG_SPLIT_K_HYBRID (-2)
/* Small-M (decode-like) kernel, for 1 <= M <= 128: each CTA computes D^T for 128 rows of B (B's
 * rows on the MMA's M side, the M rows of A on its N side, rounded up to 16), the K range of a
 * tile is split over a cluster of 1, 2 or 4 CTAs and the partial sums are added in distributed
 * shared memory, in one launch with no workspace.  BF16 or E4M3 operands (per-tensor scales),
 * BF16 or FP32 D, alpha and bias; no activation, C, gating, batches or groups.  The tile, cluster
 * and stage settings of the config do not apply (the kernel picks its own).  It is launched as a
 * programmatic dependent of the stream's previous kernel (environment CPG_DECODE_PDL=0 at plan
 * creation: not): it may start while that kernel runs, but before that kernel has completed it
 * only sets itself up and prefetches its first tiles of B into L2 (a hint, never stale data);
 * it reads A, B, the bias and the scales and writes D only after.  It lets the next kernel on
 * the stream start early in the same way. */
#define CPG_SPLIT_K_DECODE (-3)

/* Per-call epilogue options:
 *   D = act(alpha * s_a * s_b * (A . B^T) + bias + beta * C), rounded to D's type.
 * alpha scales the fp32 accumulator; scale_a / scale_b (optional device pointers to one fp32
 * value each) are the per-tensor dequantisation scales of FP8 operands; bias (optional device
 * pointer, BF16, length N) is added per column; source (optional device pointer to C, same type
 * and M x N shape as D, row stride ld_source elements, 16-byte aligned rows; it may be D itself)
 * is added times beta; activation is one of CPG_ACT_*.  The reference has none of these
 * (D = A . B^T, gemm_base.py:133); alpha = 1, NULL pointers and CPG_ACT_NONE give exactly that.
 * Activations and C need the whole K in one pass (no split-K / Stream-K). */
typedef struct cpg_epilogue {
  float alpha;
  const void* bias;
  const float* scale_a;
  const float* scale_b;
  float beta;
  int32_t activation;
  const void* source;
  int64_t ld_source;
  int64_t batch_stride_source; /* elements between the batches of C (batched problems) */
} cpg_epilogue;

#define CPG_ACT_NONE 0
#define CPG_ACT_RELU 1
#define CPG_ACT_SILU 2      /* y / (1 + exp(-y)) */
#define CPG_ACT_GELU 3      /* 0.5 y (1 + erf(y / sqrt 2)) */
#define CPG_ACT_GELU_TANH 4 /* 0.5 y (1 + tanh(sqrt(2 / pi) (y + 0.044715 y^3))) */

typedef struct cpg_gemm cpg_gemm; /* opaque compiled GEMM */

/* Reference constructor asserts (gemm_base.py:72-74, :87, :113, :122; tile_scheduler.py:51). */
int cpg_config_validate(const cpg_gemm_config* cfg);

/* Validate config + problem for this device, pick the kernel, compute scheduler params and the
 * launch grid (replaces cute.compile of GemmSM90.__call__, gemm_base.py:124-160, :608). */
int cpg_gemm_create(const cpg_gemm_config* cfg, const cpg_gemm_problem* prob, int device,
                    cpg_gemm** out);

/* Launch D = alpha * A . B^T (+ bias) on `stream` (a cudaStream_t, NULL = legacy default
 * stream).  Replaces compiled_gemm(a, b, c, stream) (gemm_base.py:609).  epi may be NULL.
 * A plan holds device state that its launches reuse (the status word; for the Stream-K fixup and
 * hybrid splits a workspace and counters; for grouped plans the tile prefix): launches of one
 * plan must be ordered on the device (one stream, or streams joined by events).  Concurrent
 * streams use one plan each; plans are independent of one another.  A plan also caches the
 * tensor maps of the last A, B, D pointers, so one host thread at a time may call it. */
int cpg_gemm_run(cpg_gemm* g, const void* a, const void* b, void* d, const cpg_epilogue* epi,
                 void* stream);

/* Grouped GEMM launch on a plan created with prob->grouped = 1: for every group g,
 *   D[r] = epilogue(A[r] . B[g]^T) for the rows r in [group_offsets[g], group_offsets[g + 1]),
 * with group_offsets a device array of G + 1 int32 (non-decreasing, within [0, m]; empty groups
 * allowed); rows of D outside every group are not written.  A small kernel turns the offsets
 * into the tile list on the device (no host synchronisation).  Offsets that break the rule make
 * their groups empty and set status 0x200 (cpg_gemm_status).  No counterpart in the reference,
 * whose kernel fixes the L mode at one (gemm_base.py:221). */
int cpg_gemm_run_grouped(cpg_gemm* plan, const void* a, const void* b, void* d,
                         const int32_t* group_offsets, const cpg_epilogue* epi, void* stream);

int cpg_gemm_destroy(cpg_gemm* g);

/* Launch shape chosen at create time: grid and cluster dims, threads per CTA, dynamic shared
 * memory bytes and the max active clusters the occupancy query returned. */
int cpg_gemm_launch_info(const cpg_gemm* g, int32_t grid[3], int32_t cluster[3],
                         int32_t* threads, int32_t* smem_bytes, int32_t* max_active_clusters);

/* Scheduler parameters of this plan. */
int cpg_gemm_sched_params(const cpg_gemm* g, cpg_sched_params* out);

/* Optional device tile trace: when set, the kernel writes (pid_m, pid_n) of the k-th tile of
 * CTA c (c = x + gx * (y + gy * z)) to buf[2 * (c * tiles_per_cta + k)].  NULL disables it. */
int cpg_gemm_set_trace(cpg_gemm* g, int32_t* device_buf, int32_t tiles_per_cta);

/* Per-wait deadline of the kernel in milliseconds (default 10000). */
int cpg_gemm_set_timeout_ms(cpg_gemm* g, int32_t timeout_ms);

/* Test hook for the kernel's bounded waits.  CPG_INJECT_SKIP_LOADS makes the next launches'
 * producer issue no loads, so the MMA warp's first wait runs out its deadline: the kernel then
 * records the wait site in the status word, stops every role, frees TMEM and returns (no GPU
 * fault, the context stays usable).  0 restores normal operation. */
#define CPG_INJECT_SKIP_LOADS 1
int cpg_gemm_set_fault_injection(cpg_gemm* g, int32_t flags);

/* Read and clear the plan's device status word (synchronises the device).  *status receives 0 or
 * 0x100 | wait-site; the return value is CPG_ERR_DEVICE_TIMEOUT when it was nonzero. */
int cpg_gemm_status(cpg_gemm* g, int32_t* status);

/* FastDivmod (fast_math.py:56-81), host side. */
int cpg_fast_divmod_create(int32_t divisor, cpg_fast_divmod* out);
int cpg_fast_divmod_divmod(const cpg_fast_divmod* f, int32_t x, int32_t* q, int32_t* r);

/* FastDivmod on the device, the kernels' own code: q[i], r[i] = divmod(x[i]) for n device values. */
int cpg_fast_divmod_device(const cpg_fast_divmod* f, const int32_t* x, int32_t* q, int32_t* r,
                           int64_t n, void* stream);

/* Scheduler (tile_scheduler.py:50-146), host side. */
int cpg_sched_params_create(int32_t ntiles_m, int32_t ntiles_n, int32_t ntiles_l,
                            int32_t raster_order, int32_t group_size, int32_t cluster_m,
                            int32_t cluster_n, int32_t cluster_k, int32_t is_persistent,
                            cpg_sched_params* out);
int cpg_sched_grid_shape(const cpg_sched_params* p, int32_t max_active_clusters, int32_t grid[3]);
/* Raster group size a plan of this config uses for K ranges of k elements of type dtype_ab: the
 * config's group_size for the static schedule; for the dynamic one the largest size up to it whose
 * re-read operand panel (AlongN: tile_n * cluster_n rows of B; AlongM: 128 * cluster_m rows of
 * A; over the K range) takes at most 32 MiB, at least 1.  No counterpart in the reference. */
int cpg_sched_plan_group_size(const cpg_gemm_config* cfg, int64_t k, int32_t dtype_ab,
                              int32_t* out);
/* out[2*i], out[2*i+1] = cluster (m, n) of linear cluster id i, for i < n. */
int cpg_sched_cluster_map(const cpg_sched_params* p, int32_t* out, int64_t n);
int cpg_sched_cluster_map_device(const cpg_sched_params* p, int32_t* device_out, int64_t n,
                                 void* stream);

/* Clusters of `cluster_size` CTAs of the default GEMM kernel that fit on the current device at
 * once (tile_scheduler.py:20-22). */
int cpg_max_active_clusters(int32_t cluster_size, int32_t* out);

/* FP8 E4M3 quantisation of x [rows, cols] (BF16 or FP32, row stride ldx) into q (row stride ldq)
 * with s = amax(|x|) / 448 per block and q = e4m3(x / s) (round to nearest even, saturating).
 * (block_rows, block_cols) = (0, 0): one scale per tensor, scales[0];
 *                            (1, 128): per row and 128 columns, scales[kb * rows + r];
 *                            (128, 128): scales[rb * ceil(cols / 128) + kb].
 * Produces the FP8 operands of the GEMM on the GPU (the reference has no FP8 path). */
int cpg_quantize_e4m3(const void* x, int32_t dtype_x, int64_t rows, int64_t cols, int64_t ldx,
                      void* q, int64_t ldq, float* scales, int32_t block_rows, int32_t block_cols,
                      void* stream);

/* y = bf16(x + bias) for x FP32 [rows, cols]: the last step of split-K after the reduction.
 * bias is optional (BF16, length cols). */
int cpg_cast_f32_bf16(const float* x, int64_t rows, int64_t cols, int64_t ldx, void* y,
                      int64_t ldy, const void* bias, void* stream);

/* Split-K GEMM with BF16 output that allocates no device memory.  No counterpart in the
 * reference: its kernel never needs scratch memory.
 *
 * Some callers cannot call cudaMalloc -- an embedding runtime whose device memory is carved up in
 * advance, or code that must not allocate while other work is being captured into a CUDA graph.
 * The split-K path (cpg_gemm_run with split_k > 1 into an FP32 D, then cpg_cast_f32_bf16) needs
 * an FP32 buffer of M x N partial sums; this entry point keeps that buffer in a 16 MiB array
 * compiled into the library (a file-scope __device__ array that every GPU loading the library
 * holds until the process exits) and writes BF16 D = alpha * s_a * s_b * A . B^T + bias.
 *   - cfg and prob as for cpg_gemm_create, with prob->dtype_d = CPG_DTYPE_BF16, scale_mode
 *     CPG_SCALE_TENSOR and split_k the number of K ranges (0 or 1: none).
 *   - The caller still passes A, B and D (device memory) and the stream; epi may be NULL.
 *   - Limit: M * round_up(N, 4) * 4 bytes <= 16 MiB (M * N <= 4,194,304); larger problems are
 *     rejected with CPG_ERR_INVALID_SHAPE and a message naming the sizes.
 *   - It calls no cudaMalloc / cudaFree.  The first call on a device looks up the array's
 *     device address (cudaGetSymbolAddress, which also loads the module there); make that first
 *     call before any stream capture.  The address is kept for the life of the process: a
 *     cudaDeviceReset unloads the module on that device and would leave it stale, so do not call
 *     this entry point on a device after resetting it.
 *   - Every call uses the same array and it keeps the last call's contents; the call clears the
 *     part it accumulates into.  Calls that overlap on the GPU (different streams, or different
 *     host threads) race on the array and must be serialised by the caller.
 *   - There is no status word: a kernel wait that runs past its deadline stops the kernel
 *     without a report (use the plan-based API when that must be observed). */
int cpg_gemm_splitk_static(const cpg_gemm_config* cfg, const cpg_gemm_problem* prob,
                           const void* a, const void* b, void* d, const cpg_epilogue* epi,
                           void* stream);

/* ---- Split-K reduce-scatter over peer memory (NVLink) -------------------------------------
 * The tall-K multi-GPU path without a separate collective: rank r multiplies its K range and
 * its GEMM's epilogue adds every FP32 partial tile straight into the buffer of the rank that
 * owns the tile's rows (system-scope atomics into the peer's memory, overlapping the next tiles'
 * math), then counts itself on that rank's arrival counter; each rank finishes its own rows with
 * cpg_peer_finish.  Replaces the NCCL reduce-scatter of the partials for ranks whose GPUs can
 * map each other's memory.  No counterpart in the reference. */
#define CPG_MAX_PEERS 8

/* Opaque inter-process handle of a peer buffer (cudaIpcMemHandle_t). */
typedef struct cpg_ipc_handle {
  uint8_t bytes[64];
} cpg_ipc_handle;

/* Zeroed device memory other processes can map: cudaMalloc + memset + an IPC handle. */
int cpg_peer_alloc(int64_t bytes, void** dev_ptr, cpg_ipc_handle* handle);
/* Map another process's cpg_peer_alloc buffer into this one (on the current device). */
int cpg_peer_open(const cpg_ipc_handle* handle, void** dev_ptr);
int cpg_peer_close(void* dev_ptr);  /* unmap a cpg_peer_open mapping */
int cpg_peer_free(void* dev_ptr);   /* free a cpg_peer_alloc buffer */

typedef struct cpg_reduce_scatter {
  int32_t ranks;                       /* 1..CPG_MAX_PEERS */
  int32_t rank;                        /* this process's rank */
  int64_t row_start[CPG_MAX_PEERS + 1]; /* rank q owns D rows [row_start[q], row_start[q + 1]):
                                          row_start[0] = 0, row_start[ranks] = M, interior
                                          boundaries multiples of 128 */
  int64_t ld;                          /* row stride (elements) of every rank's buffer, >= N,
                                          a multiple of 4 */
  float* dst[CPG_MAX_PEERS];           /* rank q's FP32 buffer ([its rows, ld], zero before the
                                          call) as mapped in this process */
  uint32_t* count[CPG_MAX_PEERS];      /* rank q's arrival counter as mapped in this process */
} cpg_reduce_scatter;

/* Run a plan (dtype_d = CPG_DTYPE_F32, split_k >= 0, no Stream-K / batches / groups / gating,
 * per-tensor scales only, N a multiple of 4) on this rank's K range, adding the partial sums
 * into the owners' buffers; epi may carry alpha and FP8 scales (no bias, activation or C). */
int cpg_gemm_run_reduce_scatter(cpg_gemm* plan, const void* a, const void* b,
                                const cpg_reduce_scatter* rs, const cpg_epilogue* epi,
                                void* stream);
/* How much one cpg_gemm_run_reduce_scatter of this plan raises each rank's counter:
 * per_rank[q] for q < rs->ranks (one per epilogue warp -- 4, or 8 for tile_n 512 -- of every
 * CTA tile whose rows rank q owns), plus one: every call also arrives once on every rank's
 * counter after its GEMM, so that each finish also waits for every rank's previous finish (a
 * rank owning no rows would otherwise not wait at all and could run two calls ahead into a
 * buffer its owner has not read yet). */
int cpg_gemm_rs_arrivals(const cpg_gemm* plan, const cpg_reduce_scatter* rs, uint32_t* per_rank);
/* The tiles' share of that count (without the call's own arrival) from scheduler parameters and
 * the tile width alone (no device needed). */
int cpg_sched_rs_arrivals(const cpg_sched_params* sched, int32_t tile_n,
                          const cpg_reduce_scatter* rs, uint32_t* per_rank);
/* Owner side: wait (bounded by timeout_ms; on a timeout *status gets a nonzero code and nothing
 * is written) until *count reaches target (modulo 2^32; the sum of every rank's arrivals on this
 * rank over all calls so far), then d = bf16(w + bias) for rows x cols and w = 0.  cols, ldw and
 * ldd multiples of 4; bias optional (BF16, length cols). */
int cpg_peer_finish(float* w, int64_t ldw, const uint32_t* count, uint32_t target, int64_t rows,
                    int64_t cols, void* d, int64_t ldd, const void* bias, int32_t* status,
                    int32_t timeout_ms, void* stream);

const char* cpg_strerror(int code);
const char* cpg_last_error_message(void);
/* ABI version, bumped on any incompatible change of this header. */
int cpg_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* CPGEMM_H_ */
