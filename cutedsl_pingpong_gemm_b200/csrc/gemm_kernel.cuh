// Warp-specialised persistent GEMM for sm_100a (BF16 or FP8 E4M3 operands, BF16 or FP32 D):
//   D[M,N] = act(alpha * s_a * s_b * A[M,K] . B[N,K]^T + bias[N] + beta * C)
//
// Role of each warp (192 threads per CTA; 512-wide tiles: 384, see EpiShape):
//   warp 0     TMA producer: one lane streams A/B k-blocks into an `ab_stages`-deep ring of
//              128B-swizzled shared-memory stages (full/empty mbarrier pairs).  This replaces the
//              reference's producer warp (gemm_base.py:204-229, produce_mainloop :365-388).
//   warp 1     MMA issuer: allocates TMEM, one lane issues tcgen05.mma (kind::f16 or
//              kind::f8f6f4, fp32 accumulate) into a TMEM accumulator and commits stage releases
//              and "accumulator full" signals.  Replaces the consumer warpgroups' wgmma mainloop
//              (consume_mainloop, gemm_base.py:390-428).  Tiles up to 256 wide keep two
//              accumulators, so the epilogue of tile i overlaps the mainloop of tile i+1; a
//              512-wide tile (two N = 256 MMAs per k-step) fills TMEM with one.
//   warps 2-5  epilogue (512-wide tiles: warps 4-11, two per quadrant, each half the columns):
//              tcgen05.ld the accumulator (each warp owns a 32-lane TMEM quadrant),
//              scale, add bias and beta * C, apply the activation (or the gated product of a
//              gate / up accumulator pair), round, write 128B-swizzled staging buffers and
//              TMA-store or TMA-reduce-add them (epilogue, gemm_base.py:270-363).
//
// CTA pairs (CtaGroup == 2, cluster (2,1)): both CTAs load their own 128 rows of A and their own
// half of the B tile; the even CTA issues tcgen05.mma.cta_group::2 (M = 256) that reads both
// CTAs' shared memory, and one tcgen05.commit with a two-CTA mask signals the same barrier in both
// CTAs.  No TMA load uses cluster multicast.
//
// Tile order: every role walks the same sequence of segments (SegmentIter): the tiles of the
// shared scheduler header, identical to the reference's SimpleTileScheduler
// (tile_scheduler.py:94-183) with its L index carrying batches and split-K ranges; Stream-K
// ranges of the (tile, k-block) space; or the tiles of a grouped GEMM's ragged groups.  With
// the dynamic schedule the same linear tile ids come from cluster launch control instead of a
// fixed stride (WorkScheduler / WorkReader below).
//
// FP32 outputs can also go to other GPUs: with rs_ranks > 0 the epilogue adds each tile into
// the buffer of the rank that owns its rows, over NVLink (the split-K reduce-scatter).
//
// Every mbarrier wait is bounded (WaitCtx): on a timeout the kernel records an error code in the
// status word, the other roles stop at their next wait, in-flight TMA loads and MMAs are drained
// (again bounded), TMEM is freed and the kernel returns.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "ptx.cuh"
#include "tile_scheduler.h"

namespace cpg {

constexpr int kBM = 128;             // rows of A / D per CTA
constexpr int kRowBytes = 128;       // one 128-byte swizzled row of a k-block
constexpr int kEpiWarps = 4;         // epilogue warps of the narrower tiles (one per TMEM quadrant)
constexpr int kEpiBufBytes = 32 * kRowBytes;  // 32 rows x 128 bytes = 4 KiB per staging buffer

// Warp layout per tile width.  Tiles up to 256 wide: 192 threads -- producer, MMA issuer and 4
// epilogue warps (warps 2-5, one per TMEM lane quadrant); the epilogue of one tile overlaps the
// next tile's mainloop through two TMEM accumulators.  512-wide tiles fill TMEM with one
// accumulator, so the next tile's MMAs wait until the epilogue has read it out; they get 8
// epilogue warps (warps 4-11, two per lane quadrant, each reading half of the columns) behind a
// warpgroup of producer, MMA issuer and 2 idle warps: 384 threads launched with 168 registers,
// the first warpgroup dropping to 56 and the epilogue warpgroups rising to 224
// (128 * 56 + 256 * 224 = 384 * 168).
template <int BN>
struct EpiShape {
  static constexpr bool kWide = BN == 512;
  static constexpr int kWarps = kWide ? 8 : 4;
  static constexpr int kFirstWarp = kWide ? 4 : 2;
  static constexpr int kThreads = (kFirstWarp + kWarps) * 32;  // 384 or 192
  static constexpr int kHalves = kWarps / 4;                   // warps per TMEM lane quadrant
  static constexpr int kLaunchRegs = 168;
  static constexpr int kLowRegs = 56;
  static constexpr int kHighRegs = 224;
  static_assert(!kWide || 128 * kLowRegs + 256 * kHighRegs == kThreads * kLaunchRegs,
                "register split must add up to the launch allocation");
};

// FP8 E4M3 storage type (one byte per element).
struct e4m3_t {
  uint8_t bits;
};

// Operand element type -> k-block width and UMMA instruction kind.
template <typename T>
struct OperandTraits;
template <>
struct OperandTraits<__nv_bfloat16> {
  static constexpr int kBK = 64;     // elements per 128-byte row
  static constexpr int kUmmaK = 16;  // K per tcgen05.mma kind::f16
  static constexpr bool kFp8 = false;
};
template <>
struct OperandTraits<e4m3_t> {
  static constexpr int kBK = 128;
  static constexpr int kUmmaK = 32;  // K per tcgen05.mma kind::f8f6f4
  static constexpr bool kFp8 = true;
};

// Output element type -> columns per 128-byte staging row.
template <typename T>
struct OutputTraits;
template <>
struct OutputTraits<__nv_bfloat16> {
  static constexpr int kStoreCols = 64;
};
template <>
struct OutputTraits<float> {
  static constexpr int kStoreCols = 32;
};
constexpr int kMaxStages = 12;
constexpr int kMaxEpiStages = 4;
constexpr int kMinSmemForOneCtaPerSm = 116 * 1024;
constexpr int kWorkSlots = 4;    // dynamic scheduling: entries of the work ring
constexpr int kMaxPeers = 8;     // reduce-scatter over peer memory: ranks
constexpr int kDynBytes = 16 * kWorkSlots + 16 + 16 + 4 * kWorkSlots;  // DynLayout

// Wait-site identifiers recorded in the status word on a timeout.
enum WaitSite : int32_t {
  kSiteProducerEmpty = 1,
  kSiteMmaFull = 2,
  kSiteMmaTmemEmpty = 3,
  kSiteEpiTmemFull = 4,
  kSiteDrainLoads = 5,
  kSiteDrainMma = 6,
  kSiteWorkFull = 7,    // dynamic scheduling: waiting for the next work entry
  kSiteWorkEmpty = 8,   // dynamic scheduling: waiting for a free work entry
  kSiteClc = 9,         // dynamic scheduling: waiting for a cluster launch control response
  kSitePeerArrivals = 10,  // peer reduce-scatter: the owner waiting for the ranks' tiles
};

struct GemmParams {
  SchedParams sched;
  int32_t m, n, k;
  int32_t k_iters;        // k-blocks of the whole K: ceil(K / BK)
  int32_t k_iters_per_split;  // k-blocks per L index (split-K); == k_iters without splitting
  int32_t reduce_add;     // epilogue adds into D (fp32 split-K partial sums) instead of storing
  int32_t stream_k;       // persistent CTAs split the (tile, k-block) space evenly (Stream-K)
  int32_t ab_stages;
  int32_t epi_stages;
  int32_t reuse_ab;       // epilogue staging aliases the A/B stages (single-tile CTAs only)
  float alpha;
  const float* scale_a;   // optional device scalar (FP8 per-tensor scale of A); D *= *scale_a
  const float* scale_b;   // optional device scalar (FP8 per-tensor scale of B)
  const __nv_bfloat16* bias;  // optional per-column bias, length N
  int32_t* tile_trace;    // optional: (pid_m, pid_n) per CTA per tile, trace_stride tiles per CTA
  int32_t trace_stride;
  int32_t* status;        // device status word (0 = ok)
  uint64_t timeout_ns;
  int32_t fault_inject;   // test hook: kInjectSkipLoads makes the producer issue no loads
  int32_t l2_policy_a;    // L2 eviction priority of A / B tile loads: 0 normal, 1 first, 2 last
  int32_t l2_policy_b;
  int32_t l2_policy_d;    // ... of the D tile stores (D is written once and not read back)
  // Fused epilogue: D = act(alpha * acc + bias + beta * C); gated (512-wide tiles only):
  // D[:, n] = act(alpha * acc_gate[:, n]) * alpha * acc_up[:, n] with B = [W_gate; W_up].
  int32_t act;            // kActNone, kActRelu, kActSilu, kActGelu, kActGeluTanh
  float beta;
  const void* src;        // optional C, same type and shape as D
  int64_t ld_src;         // row stride of C, elements
  int64_t src_batch_stride;  // elements between the batches of C
  int32_t gated;
  // The scheduler's L index is batch * num_splits + split (split-K ranges of each batch).
  int32_t num_splits;
  // Grouped GEMM (ragged groups, MoE-style; GroupInfo): group g owns rows
  // [group_offsets[g], group_offsets[g + 1]) of A and D and batch g of B.
  int32_t num_groups;             // 0: not grouped
  const int32_t* group_offsets;   // [num_groups + 1], device
  const int32_t* tile_prefix;     // [num_groups + 1]: cluster tiles of the groups before g
  int32_t group_n_clusters;       // cluster columns of every group
  void* d;                        // D itself: rows at a group boundary are stored per thread
  int64_t ldd;
  // Stream-K with in-kernel fixup (stream_k != 0 and fixup != 0): the first dp_tiles cluster
  // tiles are computed whole (data-parallel waves, persistent stride), the k-blocks of the
  // others are shared evenly by the clusters.  A segment that covers only part of a tile adds
  // alpha * acc into that CTA's FP32 workspace tile (tm_ws, rows (cid - dp_tiles) * ctas + rank)
  // and counts its k-blocks in fixup_count; the segment that completes the count rounds the
  // tile (+ bias) into D and clears the workspace tile and its count for the next launch.
  int32_t fixup;
  int32_t dp_tiles;
  int32_t* fixup_count;           // [sk tiles * CTAs per cluster], zero between launches
  float* fixup_ws;                // FP32 workspace the fixup reads (and clears)
  int32_t ws_cols;                // row length of a workspace tile (the tile's output columns)
  // Dynamic scheduling (cluster launch control, WorkScheduler): the grid holds one cluster per
  // cluster tile along x and running clusters take over clusters that have not started.
  int32_t dynamic;
  // Reduce-scatter over peer memory (rs_ranks > 0): every segment adds alpha * acc into the FP32
  // buffer of the rank that owns its rows (rows [rs_row_start[q], rs_row_start[q + 1]) belong to
  // rank q, stored from row 0 of rs_dst[q] with row stride rs_ld), with system-scope atomics
  // over NVLink, then each epilogue warp counts itself on the owner's rs_count (release).
  int32_t rs_ranks;
  int32_t rs_row_start[kMaxPeers + 1];
  int64_t rs_ld;
  float* rs_dst[kMaxPeers];
  uint32_t* rs_count[kMaxPeers];
};

// The grouped mode of the segment iterator (num_groups == 0: the scheduler's tiles).
struct GroupInfo {
  int32_t num_groups;
  const int32_t* offsets;
  const int32_t* prefix;
  int32_t n_clusters;
};

__device__ __forceinline__ GroupInfo group_info(const GemmParams& p) {
  return GroupInfo{p.num_groups, p.group_offsets, p.tile_prefix, p.group_n_clusters};
}

enum Activation : int32_t {
  kActNone = 0,
  kActRelu = 1,
  kActSilu = 2,
  kActGelu = 3,      // 0.5 y (1 + erf(y / sqrt(2)))
  kActGeluTanh = 4,  // 0.5 y (1 + tanh(sqrt(2 / pi) (y + 0.044715 y^3)))
};

__device__ __forceinline__ float act_relu(float y) { return fmaxf(y, 0.f); }
// y / (1 + e^-y); the fast divide returns 0 once e^-y passes 2^126, the limit of silu there.
__device__ __forceinline__ float act_silu(float y) { return __fdividef(y, 1.f + __expf(-y)); }
__device__ __forceinline__ float act_gelu(float y) {
  return 0.5f * y * (1.f + erff(y * 0.70710678118654752f));
}
__device__ __forceinline__ float act_gelu_tanh(float y) {
  return 0.5f * y * (1.f + tanhf(0.79788456080286536f * (y + 0.044715f * y * y * y)));
}

// x[j] = act(x[j]).  The switch sits outside the unrolled loops, so each activation's code is
// one contiguous block (a switch per element would interleave all four bodies N times).
template <int N>
__device__ __forceinline__ void act_inplace(int32_t act, float (&x)[N]) {
  switch (act) {
    case kActRelu:
#pragma unroll
      for (int j = 0; j < N; ++j) x[j] = act_relu(x[j]);
      break;
    case kActSilu:
#pragma unroll
      for (int j = 0; j < N; ++j) x[j] = act_silu(x[j]);
      break;
    case kActGelu:
#pragma unroll
      for (int j = 0; j < N; ++j) x[j] = act_gelu(x[j]);
      break;
    case kActGeluTanh:
#pragma unroll
      for (int j = 0; j < N; ++j) x[j] = act_gelu_tanh(x[j]);
      break;
    default:
      break;
  }
}

// Host-selected fault injection for testing the bounded waits: with kInjectSkipLoads the
// producer issues nothing, so the MMA warp's first `full` wait must run out its deadline.
constexpr int32_t kInjectSkipLoads = 1;

template <int BN, int CtaGroup>
struct GemmSmem {
  static constexpr int kAStageBytes = kBM * kRowBytes;                     // 16 KiB
  static constexpr int kBStageBytes = (BN / CtaGroup) * kRowBytes;         // per CTA
  static constexpr int kStageBytes = kAStageBytes + kBStageBytes;
  // tcgen05.mma takes N <= 256: a 512-wide tile issues two MMAs per k-step and keeps a single
  // accumulator (512 TMEM columns); narrower tiles keep two accumulators so that the epilogue of
  // one tile overlaps the mainloop of the next.
  static constexpr int kMmaN = BN > 256 ? 256 : BN;                        // N of one MMA
  static constexpr int kNumMma = BN / kMmaN;                               // MMAs per k-step
  static constexpr int kBRowsPerMma = kMmaN / CtaGroup;                    // B rows per CTA
  static constexpr int kAccStages = 2 * BN <= 512 ? 2 : 1;
  static constexpr int kTmemCols = kAccStages * BN;
  static_assert(kStageBytes % 1024 == 0, "stages must keep 1024-byte alignment");
  static_assert(kTmemCols >= 32 && kTmemCols <= 512 && (kTmemCols & (kTmemCols - 1)) == 0,
                "TMEM allocation must be a power of two in [32, 512]");

  // Byte offsets from the 1024-aligned base.
  static __host__ __device__ int epi_offset(int stages, int reuse_ab) {
    return reuse_ab ? 0 : stages * kStageBytes;
  }
  static __host__ __device__ int barrier_offset(int stages, int epi_stages, int reuse_ab) {
    int end_stages = stages * kStageBytes;
    int end_epi = epi_offset(stages, reuse_ab) + EpiShape<BN>::kWarps * epi_stages * kEpiBufBytes;
    return end_stages > end_epi ? end_stages : end_epi;
  }
  // full[S], empty[S], tmem_full[2], tmem_empty[2], drain[1]; then tmem slot and abort flag;
  // then (16-byte aligned) the dynamic scheduler's kDynBytes (DynLayout).
  static __host__ __device__ int dyn_offset(int stages, int epi_stages, int reuse_ab) {
    return (barrier_offset(stages, epi_stages, reuse_ab) + (2 * stages + 5) * 8 + 16 + 15) & ~15;
  }
  static __host__ __device__ int bytes(int stages, int epi_stages, int reuse_ab) {
    int b = dyn_offset(stages, epi_stages, reuse_ab) + kDynBytes;
    b += 1024;  // alignment slack for the dynamic shared memory base
    return b < kMinSmemForOneCtaPerSm ? kMinSmemForOneCtaPerSm : b;
  }
};

// Linear persistent / non-persistent work iterator (tile_scheduler.py:94-107, :159-183).
struct WorkIter {
  int32_t cid, stride, total, executed, persistent;
  __device__ __forceinline__ bool valid() const {
    return persistent ? (cid < total) : (executed == 0);
  }
  __device__ __forceinline__ void advance() {
    if (persistent) cid += stride;
    ++executed;
  }
};

__device__ __forceinline__ WorkIter make_work_iter(const SchedParams& sp) {
  WorkIter it;
  if (sp.is_persistent) {
    it.cid = static_cast<int32_t>(blockIdx.z);
    it.stride = static_cast<int32_t>(gridDim.z);
  } else {
    // tile_scheduler.py:100-102 (clusterid.x + clusterid.y * nclusterid.x), extended by the
    // grid's z (the L index) so that L > 1 launches cover every (tile, L) pair once.
    it.cid = static_cast<int32_t>(ptx::clusterid_x() +
                                  ptx::nclusterid_x() * (ptx::clusterid_y() +
                                                         ptx::nclusterid_y() * ptx::clusterid_z()));
    it.stride = 0;
  }
  it.total = sched_total_clusters(sp);
  it.executed = 0;
  it.persistent = sp.is_persistent;
  return it;
}

// Linear cluster id -> (pid_m, pid_n, l).  The id is first split into the L index and the id
// within one problem with the reference's dm_clusters_per_problem (tile_scheduler.py:70, which
// the reference computes but never applies); for L = 1 this is the identity and the map is the
// reference's _map_cta_coords (tile_scheduler.py:125-146).
__device__ __forceinline__ void work_tile_coords(const SchedParams& sp, int32_t cid,
                                                 int32_t& pid_m, int32_t& pid_n, int32_t& l) {
  int32_t cid_in_problem, cm, cn;
  fast_divmod(sp.dm_clusters_per_problem, cid, l, cid_in_problem);
  sched_map_cluster(sp, cid_in_problem, cm, cn);
  pid_m = cm * sp.cluster_m + static_cast<int32_t>(ptx::cluster_ctaid_x());
  pid_n = cn * sp.cluster_n + static_cast<int32_t>(ptx::cluster_ctaid_y());
}

__device__ __forceinline__ void work_tile_coords(const SchedParams& sp, int32_t cid,
                                                 int32_t& pid_m, int32_t& pid_n) {
  int32_t l;
  work_tile_coords(sp, cid, pid_m, pid_n, l);
}

// One unit of work of a CTA: k-blocks [kb0, kb1) of the tile at linear cluster id `cid`.
struct Segment {
  int32_t cid;
  int32_t kb0, kb1;
  int32_t pid_m, pid_n;   // this CTA's tile
  int32_t batch;          // L index of the batched GEMM / group of a grouped GEMM (else 0)
  int32_t ab_batch;       // TMA batch coordinate of A and D (a grouped A / D has one batch)
  int32_t row_base;       // first row of A / D of the tile's problem (group), and its end
  int32_t row_end;
  int32_t index;          // how many segments this CTA produced before this one
};

// Walks this CTA's segments.  Tile mode: the scheduler's tiles, one segment per tile; the L
// index l = batch * splits + split selects the batch and, for split-K, the k-blocks
// [split * kps, (split + 1) * kps).  Stream-K: the linearised (tile, k-block) space of
// tiles * k_iters k-blocks (tiles of all batches) is cut into gridDim.z equal ranges and cluster
// z walks range z, one segment per tile it touches; the tiles keep the reference's
// linear-id -> (m, n, l) map.
struct SegmentIter {
  WorkIter it;
  int64_t pos, end;
  int32_t k_iters, kps, stream, index, splits;
  GroupInfo gi;
  int32_t group_total;  // cluster tiles of all groups (grouped mode)
  int32_t dp_tiles;     // Stream-K: leading cluster tiles computed whole (persistent stride)

  __device__ __forceinline__ bool next(const SchedParams& sp, Segment& s) {
    if (gi.num_groups > 0) {
      // Grouped: linear cluster tile -> group (binary search of the tile prefix) -> m-fastest
      // order inside the group, so the group's row tiles share each column tile of B in L2.
      if (it.cid >= group_total) return false;
      const int32_t cid = it.cid;
      int32_t lo = 0, hi = gi.num_groups;
      while (hi - lo > 1) {
        const int32_t mid = (lo + hi) >> 1;
        if (gi.prefix[mid] <= cid) lo = mid; else hi = mid;
      }
      const int32_t local = cid - gi.prefix[lo];
      const int32_t count = gi.prefix[lo + 1] - gi.prefix[lo];
      const int32_t m_clusters = count / gi.n_clusters;
      const int32_t cm = local % m_clusters, cn = local / m_clusters;
      s.cid = cid;
      s.kb0 = 0;
      s.kb1 = k_iters;
      s.pid_m = cm * sp.cluster_m + static_cast<int32_t>(ptx::cluster_ctaid_x());
      s.pid_n = cn * sp.cluster_n + static_cast<int32_t>(ptx::cluster_ctaid_y());
      s.batch = lo;
      s.ab_batch = 0;
      s.row_base = gi.offsets[lo];
      s.row_end = gi.offsets[lo + 1];
      it.cid += it.stride;
      s.index = index++;
      return true;
    }
    s.row_base = 0;
    s.row_end = 0x7fffffff;
    if (stream && it.cid < dp_tiles) {
      // Data-parallel waves before the Stream-K tail: whole tiles in the persistent order.
      s.cid = it.cid;
      s.kb0 = 0;
      s.kb1 = k_iters;
      int32_t l, cid_in_problem;
      fast_divmod(sp.dm_clusters_per_problem, s.cid, l, cid_in_problem);
      s.batch = l;
      s.ab_batch = l;
      work_tile_coords(sp, s.cid, s.pid_m, s.pid_n);
      it.cid += it.stride;
      s.index = index++;
      return true;
    }
    if (stream) {
      if (pos >= end) return false;
      const int64_t tile = pos / k_iters;
      const int32_t kb0 = static_cast<int32_t>(pos - tile * k_iters);
      int64_t kb1 = kb0 + (end - pos);
      if (kb1 > k_iters) kb1 = k_iters;
      s.cid = static_cast<int32_t>(tile);
      s.kb0 = kb0;
      s.kb1 = static_cast<int32_t>(kb1);
      int32_t l, cid_in_problem;
      fast_divmod(sp.dm_clusters_per_problem, s.cid, l, cid_in_problem);
      s.batch = l;
      s.ab_batch = l;
      work_tile_coords(sp, s.cid, s.pid_m, s.pid_n);
      pos += kb1 - kb0;
    } else {
      if (!it.valid()) return false;
      int32_t l, cid_in_problem;
      fast_divmod(sp.dm_clusters_per_problem, it.cid, l, cid_in_problem);
      const int32_t batch = splits > 1 ? l / splits : l;
      s.cid = it.cid;
      s.batch = batch;
      s.ab_batch = batch;
      s.kb0 = (l - batch * splits) * kps;
      s.kb1 = s.kb0 + kps < k_iters ? s.kb0 + kps : k_iters;
      work_tile_coords(sp, s.cid, s.pid_m, s.pid_n);
      it.advance();
    }
    s.index = index++;
    return true;
  }
};

__device__ __forceinline__ SegmentIter make_segment_iter(const SchedParams& sp, int32_t k_iters,
                                                         int32_t kps, int32_t stream_k,
                                                         int32_t splits,
                                                         GroupInfo gi = GroupInfo{0, nullptr,
                                                                                  nullptr, 1},
                                                         int32_t dp_tiles = 0,
                                                         int32_t dynamic = 0) {
  SegmentIter si;
  si.it = make_work_iter(sp);
  // Dynamic scheduling sets it.cid before every next(); a tile is valid below the total.
  if (dynamic) si.it.persistent = 1;
  si.gi = gi;
  si.dp_tiles = stream_k ? dp_tiles : 0;
  si.group_total = gi.num_groups > 0 ? gi.prefix[gi.num_groups] : 0;
  si.k_iters = k_iters;
  si.kps = kps;
  si.stream = stream_k;
  si.splits = splits > 1 ? splits : 1;
  si.index = 0;
  si.pos = si.end = 0;
  if (stream_k) {
    const int64_t base = static_cast<int64_t>(si.dp_tiles) * k_iters;
    const int64_t total = static_cast<int64_t>(sched_total_clusters(sp)) * k_iters - base;
    const int64_t z = blockIdx.z, g = gridDim.z;
    si.pos = base + total * z / g;
    si.end = base + total * (z + 1) / g;
  }
  return si;
}

__device__ __forceinline__ void epi_wait_buffer(int epi_stages) {
  // Allow (epi_stages - 1) stores in flight before reusing the oldest staging buffer.
  switch (epi_stages) {
    case 1: ptx::bulk_wait_group_read<0>(); break;
    case 2: ptx::bulk_wait_group_read<1>(); break;
    case 3: ptx::bulk_wait_group_read<2>(); break;
    default: ptx::bulk_wait_group_read<3>(); break;
  }
}

// This thread's 128-byte chunk of row `row` of the C source from column col0, as raw words;
// elements outside C read as zero.
template <typename OutT>
__device__ __forceinline__ void load_row_chunk(const GemmParams& p, int32_t batch, int32_t row,
                                               int32_t col0, uint4 (&cs)[8]) {
  constexpr int kCols = 128 / static_cast<int>(sizeof(OutT));
  constexpr int kPer = 16 / static_cast<int>(sizeof(OutT));  // elements per 16 bytes
  const OutT* base = static_cast<const OutT*>(p.src) + batch * p.src_batch_stride +
                     static_cast<int64_t>(row) * p.ld_src + col0;
  if (row < p.m && col0 + kCols <= p.n) {
#pragma unroll
    for (int q = 0; q < 8; ++q) cs[q] = ptx::ld_global_nc_v4(base + q * kPer);
    return;
  }
  const bool row_ok = row < p.m;
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (sizeof(OutT) == 2) {
        const uint16_t* b16 = reinterpret_cast<const uint16_t*>(base) + q * 8 + 2 * i;
        const int32_t c = col0 + q * 8 + 2 * i;
        const uint32_t lo = (row_ok && c < p.n) ? b16[0] : 0u;
        const uint32_t hi = (row_ok && c + 1 < p.n) ? b16[1] : 0u;
        w[i] = lo | (hi << 16);
      } else {
        const int32_t c = col0 + q * 4 + i;
        w[i] = (row_ok && c < p.n) ? reinterpret_cast<const uint32_t*>(base)[q * 4 + i] : 0u;
      }
    }
    cs[q] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// Store this thread's 128-byte output chunk (packed BF16 pairs or FP32 words, row order) to
// row `row` of D from column col0, if row < row_end; columns past N are not written.
template <typename OutT>
__device__ __forceinline__ void store_row_chunk(const GemmParams& p, int32_t row, int32_t row_end,
                                                int32_t col0, const uint32_t (&packed)[32]) {
  if (row >= row_end) return;
  constexpr int kCols = 128 / static_cast<int>(sizeof(OutT));
  uint32_t* base = reinterpret_cast<uint32_t*>(static_cast<OutT*>(p.d) +
                                               static_cast<int64_t>(row) * p.ldd + col0);
  if (col0 + kCols <= p.n) {
#pragma unroll
    for (int q = 0; q < 8; ++q)
      ptx::st_global_v4(base + 4 * q, packed[4 * q], packed[4 * q + 1], packed[4 * q + 2],
                        packed[4 * q + 3]);
    return;
  }
  if constexpr (sizeof(OutT) == 2) {
    uint16_t* b16 = reinterpret_cast<uint16_t*>(base);
#pragma unroll
    for (int j = 0; j < kCols; ++j)
      if (col0 + j < p.n) b16[j] = static_cast<uint16_t>(packed[j >> 1] >> (16 * (j & 1)));
  } else {
#pragma unroll
    for (int j = 0; j < kCols; ++j)
      if (col0 + j < p.n) base[j] = packed[j];
  }
}

// x[j] += beta * C[j] for the 128-byte chunk of raw words from load_row_chunk.
template <typename OutT>
__device__ __forceinline__ void add_row_chunk(float beta, const uint4 (&cs)[8],
                                              float (&x)[128 / sizeof(OutT)]) {
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const uint32_t w[4] = {cs[q].x, cs[q].y, cs[q].z, cs[q].w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (sizeof(OutT) == 2) {
        x[q * 8 + 2 * i] += beta * __uint_as_float(w[i] << 16);
        x[q * 8 + 2 * i + 1] += beta * __uint_as_float(w[i] & 0xffff0000u);
      } else {
        x[q * 4 + i] += beta * __uint_as_float(w[i]);
      }
    }
  }
}

// L2 eviction priority for a TMA load: 0 normal, 1 evict-first, 2 evict-last.
__device__ __forceinline__ uint64_t l2_policy(int32_t which) {
  return which == 1 ? ptx::policy_evict_first()
                    : (which == 2 ? ptx::policy_evict_last() : ptx::policy_evict_normal());
}

// ------------------------------------------------------------------ dynamic scheduling
// Cluster launch control.  The grid holds one cluster per cluster tile (x = tile * cluster_m).
// A cluster starts with its own tile (%clusterid.x) and then takes over clusters of the grid that
// have not started: the producer lane of CTA 0 asks for one (clusterlaunchcontrol.try_cancel)
// when it starts loading a tile and, once that tile's loads are issued, publishes the answer --
// the cancelled cluster's tile, or -1 when none was left -- to every CTA of the cluster through a
// ring of kWorkSlots entries in shared memory.  full[i] of a CTA completes when its entry i is
// written (CTA 0 stores it, by distributed shared memory for the other CTAs, and arrives with
// cluster-scope release); empty[i] of CTA 0 completes when every consumer of the cluster has read
// entry i: the producer lanes of the other CTAs, the MMA lanes and the four epilogue warps of
// every CTA.  Tiles keep the scheduler's linear-id -> (m, n, l) map; only which cluster runs a
// tile is decided at run time, so CTAs that start late (SMs busy with other work) take fewer.
struct DynLayout {
  uint32_t full;      // mbarrier[kWorkSlots]
  uint32_t empty;     // mbarrier[kWorkSlots], used in CTA 0
  uint32_t clc_bar;   // mbarrier of the cluster launch control response
  uint32_t clc_resp;  // 16-byte response
  uint32_t cids;      // int32[kWorkSlots]
};

__device__ __forceinline__ DynLayout dyn_layout(uint32_t base) {
  return DynLayout{base, base + 8u * kWorkSlots, base + 16u * kWorkSlots,
                   base + 16u * kWorkSlots + 16u, base + 16u * kWorkSlots + 32u};
}

// Readers of the work ring per CTA: its producer lane (CTAs other than 0), its MMA lane (CTAs
// that issue MMAs) and its epilogue warps.
__device__ __forceinline__ uint32_t dyn_consumers(int32_t cluster_ctas, int32_t cta_group,
                                                  int32_t epi_warps) {
  return static_cast<uint32_t>(cluster_ctas * epi_warps + (cluster_ctas - 1) +
                               cluster_ctas / cta_group);
}

// A consumer's view: its own tile first, then the ring's entries in order.  CTA 0 addresses
// its own barriers by their shared::cta address (part of the shared::cluster window), so a grid
// without clusters needs no mapa.
struct WorkReader {
  DynLayout l;
  int slot;
  uint32_t phase;
  bool first;
  uint32_t rank;
  __device__ __forceinline__ WorkReader(const DynLayout& layout, uint32_t cta_rank)
      : l(layout), slot(0), phase(0), first(true), rank(cta_rank) {}
  // False on a timeout (recorded in the status word); cid = -1 when no work is left.
  __device__ __forceinline__ bool next(int32_t& cid, const ptx::WaitCtx& ctx) {
    if (first) {
      first = false;
      cid = static_cast<int32_t>(ptx::clusterid_x());
      return true;
    }
    if (!ptx::mbar_wait_acquire_cluster(l.full + 8u * slot, phase, ctx, kSiteWorkFull))
      return false;
    cid = static_cast<int32_t>(ptx::ld_shared_u32(l.cids + 4u * slot));
    const uint32_t e = l.empty + 8u * slot;
    ptx::mbar_arrive_release_cluster(rank == 0 ? e : ptx::mapa_shared(e, 0));
    if (++slot == kWorkSlots) {
      slot = 0;
      phase ^= 1u;
    }
    return true;
  }
};

// CTA 0's producer lane: requests clusters and publishes the answers.
struct WorkScheduler {
  DynLayout l;
  int slot;
  uint32_t phase, clc_phase;
  bool live, pending;
  int32_t cluster_ctas, cluster_m;
  __device__ __forceinline__ WorkScheduler(const DynLayout& layout, int32_t ctas, int32_t cm)
      : l(layout), slot(0), phase(0), clc_phase(0), live(true), pending(false),
        cluster_ctas(ctas), cluster_m(cm) {}
  __device__ __forceinline__ void request() {
    if (!live || pending) return;
    ptx::mbar_arrive_expect_tx(l.clc_bar, 16u);
    ptx::clc_try_cancel(l.clc_resp, l.clc_bar);
    pending = true;
  }
  // The answer to the outstanding request (-1: none left, or no request outstanding).
  __device__ __forceinline__ bool answer(int32_t& cid, const ptx::WaitCtx& ctx) {
    cid = -1;
    if (!pending) return true;
    if (!ptx::mbar_wait(l.clc_bar, clc_phase, ctx, kSiteClc)) return false;
    pending = false;
    clc_phase ^= 1u;
    const int32_t x = ptx::clc_query_first_x(l.clc_resp);
    ptx::fence_proxy_async_shared();  // this read before the next request's async write
    if (x < 0) {
      live = false;  // no request may follow a failed one
    } else {
      cid = x / cluster_m;
    }
    return true;
  }
  __device__ __forceinline__ bool publish(int32_t cid, const ptx::WaitCtx& ctx) {
    if (!ptx::mbar_wait_acquire_cluster(l.empty + 8u * slot, phase ^ 1u, ctx, kSiteWorkEmpty))
      return false;
    for (int32_t r = 0; r < cluster_ctas; ++r) {
      const uint32_t rr = static_cast<uint32_t>(r);
      const uint32_t c = l.cids + 4u * slot, f = l.full + 8u * slot;
      ptx::st_shared_cluster_u32(r == 0 ? c : ptx::mapa_shared(c, rr), static_cast<uint32_t>(cid));
      ptx::mbar_arrive_release_cluster(r == 0 ? f : ptx::mapa_shared(f, rr));
    }
    if (++slot == kWorkSlots) {
      slot = 0;
      phase ^= 1u;
    }
    return true;
  }
  // Before the CTA exits: a response still in flight must land in shared memory first.
  __device__ __forceinline__ void drain(const ptx::WaitCtx& ctx) {
    if (!pending) return;
    ptx::WaitCtx dctx{ctx.abort_flag, ctx.status, ctx.timeout_ns};
    volatile int32_t no_abort = 0;
    dctx.abort_flag = &no_abort;
    if (ptx::mbar_wait(l.clc_bar, clc_phase, dctx, kSiteClc)) pending = false;
  }
};

// What the roles need to know of the dynamic mode.
struct DynArgs {
  int32_t enabled;
  DynLayout layout;
  int32_t cluster_ctas;
  int32_t cluster_m;
  uint32_t rank;  // %cluster_ctarank
};

// The cluster tiles of a role that walks whole tiles: the static WorkIter, or the work ring.
// With `broadcast`, lane 0 reads the ring and the warp shares the entry (all lanes must call).
struct TileSource {
  WorkIter it;
  WorkReader reader;
  bool dynamic, started;
  __device__ __forceinline__ TileSource(const SchedParams& sp, const DynArgs& dyn)
      : it(make_work_iter(sp)), reader(dyn.layout, dyn.rank), dynamic(dyn.enabled != 0),
        started(false) {}
  // False at the end, or on a timeout (then `ok` is cleared).
  __device__ __forceinline__ bool next(int32_t& cid, const ptx::WaitCtx& ctx, bool& ok,
                                       bool broadcast) {
    if (!dynamic) {
      if (started) it.advance();
      started = true;
      if (!it.valid()) return false;
      cid = it.cid;
      return true;
    }
    int32_t got = 1;
    cid = 0;
    if (!broadcast || ptx::lane_id() == 0) got = reader.next(cid, ctx) ? 1 : 0;
    if (broadcast) {
      cid = __shfl_sync(0xffffffffu, cid, 0);
      got = __shfl_sync(0xffffffffu, got, 0);
    }
    if (!got) {
      ok = false;
      return false;
    }
    return cid >= 0;
  }
};

// TMA producer (one lane): streams the k-blocks of A (128 rows) and B (BN / CtaGroup rows) of
// every tile of this CTA into the shared-memory stage ring, then drains its in-flight loads.
// B is loaded as BN / kMmaN slots, one per MMA of width kMmaN.
template <int BN, int CtaGroup, int kBK, int kStageBytes, int kAStageBytes,
          int kMmaN = (BN > 256 ? 256 : BN)>
__device__ __forceinline__ void producer_loop(const CUtensorMap* tm_a, const CUtensorMap* tm_b,
                                              const SchedParams& sp, int k_iters,
                                              int k_iters_per_split, int stages,
                                              uint32_t base, uint32_t full_bar, uint32_t empty_bar,
                                              uint32_t rank, bool leader,
                                              const ptx::WaitCtx& ctx, int32_t l2_a = 0,
                                              int32_t l2_b = 0, int32_t stream_k = 0,
                                              int32_t b_slot_rows = 0, int32_t splits = 1,
                                              GroupInfo gi = GroupInfo{0, nullptr, nullptr, 1},
                                              int32_t dp_tiles = 0,
                                              DynArgs dyn = DynArgs{}) {
  constexpr int kNumMma = BN / kMmaN;
  constexpr int kBRowsPerMma = kMmaN / CtaGroup;
  constexpr uint32_t kTxBytes = static_cast<uint32_t>(kStageBytes * CtaGroup);
  const uint32_t leader_rank = rank & ~1u;
  volatile int32_t* abort_flag = ctx.abort_flag;
  const uint64_t pol_a = l2_policy(l2_a);
  const uint64_t pol_b = l2_policy(l2_b);
  int stage = 0;
  uint32_t phase = 0;
  uint32_t fills = 0;
  bool ok = true;
  SegmentIter si = make_segment_iter(sp, k_iters, k_iters_per_split, stream_k, splits, gi,
                                     dp_tiles, dyn.enabled);
  // Dynamic mode: CTA 0 schedules (and needs no reader), the other CTAs read the ring.
  const bool scheduler = dyn.enabled && dyn.rank == 0;
  WorkScheduler sched(dyn.layout, dyn.cluster_ctas, dyn.cluster_m);
  WorkReader reader(dyn.layout, dyn.rank);
  const int32_t valid_tiles = gi.num_groups > 0 ? si.group_total : 0x7fffffff;
  bool first = true;
  auto fetch = [&](Segment& out) -> bool {
    if (!dyn.enabled) return si.next(sp, out);
    int32_t cid;
    if (scheduler) {
      if (first) {
        first = false;
        cid = static_cast<int32_t>(ptx::clusterid_x());
        if (cid >= valid_tiles) {  // an empty cluster of a grouped GEMM's bound
          sched.publish(-1, ctx);
          return false;
        }
      } else {
        // The answer to the request made when the previous tile started; clusters past the
        // grouped GEMM's tiles are skipped by asking again.
        while (true) {
          if (!sched.answer(cid, ctx)) {
            ok = false;
            sched.publish(-1, ctx);
            return false;
          }
          if (cid < valid_tiles) break;
          sched.request();
        }
        if (!sched.publish(cid, ctx)) {
          ok = false;
          return false;
        }
        if (cid < 0) return false;
      }
      sched.request();  // for the tile after this one, answered while this one loads
    } else {
      if (!reader.next(cid, ctx)) {
        ok = false;
        return false;
      }
      if (cid < 0) return false;
    }
    si.it.cid = cid;
    return si.next(sp, out);
  };
  Segment sg;
  while (ok && fetch(sg)) {
    const int32_t pid_m = sg.pid_m, pid_n = sg.pid_n;
    const int32_t a_row = sg.row_base + pid_m * kBM;
    // B rows of MMA j: [pid_n * BN + j * kMmaN, +kMmaN), of which this CTA of a pair loads its
    // half (kBRowsPerMma rows at offset rank * kBRowsPerMma) into smem slot j.  Gated tiles
    // (b_slot_rows = N > 0) take MMA j's rows from the j-th of the stacked [W_gate; W_up]:
    // [j * N + pid_n * kMmaN, +kMmaN).
    const int32_t tile_rows = b_slot_rows > 0 ? kMmaN : BN;
    const int32_t slot_rows = b_slot_rows > 0 ? b_slot_rows : kMmaN;
    const int32_t b_row = pid_n * tile_rows + static_cast<int32_t>(rank & 1u) * kBRowsPerMma;
    for (int kb = sg.kb0; kb < sg.kb1; ++kb) {
      if (!ptx::mbar_wait(empty_bar + 8u * stage, phase ^ 1u, ctx, kSiteProducerEmpty)) {
        ok = false;
        break;
      }
      const uint32_t sa = base + static_cast<uint32_t>(stage * kStageBytes);
      const uint32_t sb = sa + kAStageBytes;
      const uint32_t fb = full_bar + 8u * stage;
      if constexpr (CtaGroup == 1) {
        ptx::mbar_arrive_expect_tx(fb, kTxBytes);
        ptx::tma_load_3d(tm_a, sa, fb, kb * kBK, a_row, sg.ab_batch, pol_a);
#pragma unroll
        for (int j = 0; j < kNumMma; ++j)
          ptx::tma_load_3d(tm_b, sb + j * kBRowsPerMma * 128, fb, kb * kBK, b_row + j * slot_rows,
                           sg.batch, pol_b);
      } else {
        if (leader) ptx::mbar_arrive_expect_tx(fb, kTxBytes);
        const uint32_t fb_leader = ptx::mapa_shared(fb, leader_rank);
        ptx::tma_load_3d_pair(tm_a, sa, fb_leader, kb * kBK, a_row, sg.ab_batch, pol_a);
#pragma unroll
        for (int j = 0; j < kNumMma; ++j)
          ptx::tma_load_3d_pair(tm_b, sb + j * kBRowsPerMma * 128, fb_leader, kb * kBK,
                                b_row + j * slot_rows, sg.batch, pol_b);
      }
      ++fills;
      if (++stage == stages) {
        stage = 0;
        phase ^= 1u;
      }
    }
  }
  if (scheduler) {
    // Error paths: finish the ring (consumers stop at -1) and let a pending response land.
    if (!ok) sched.publish(-1, ctx);
    sched.drain(ctx);
  }
  // Drain: wait (bounded) until every issued fill has landed so no TMA write into this CTA's
  // shared memory is outstanding when the CTA exits.  Immediate on the normal path.
  if (leader) {
    for (int s = 0; s < stages; ++s) {
      if (fills > static_cast<uint32_t>(s)) {
        const uint32_t round = (fills - 1u - static_cast<uint32_t>(s)) / stages;
        ptx::WaitCtx dctx{abort_flag, ctx.status, ctx.timeout_ns};
        volatile int32_t no_abort = 0;
        dctx.abort_flag = &no_abort;
        ptx::mbar_wait(full_bar + 8u * s, round & 1u, dctx, kSiteDrainLoads);
      }
    }
  } else {
    // The peer's loads complete on the leader's barriers; the leader drains them, and the
    // final cluster barrier keeps this CTA resident until then.  Waiting for the stage to be
    // released covers loads whose consumer never ran.
    for (int s = 0; s < stages; ++s) {
      if (fills > static_cast<uint32_t>(s)) {
        const uint32_t round = (fills - 1u - static_cast<uint32_t>(s)) / stages;
        ptx::WaitCtx dctx{abort_flag, ctx.status, ctx.timeout_ns};
        volatile int32_t no_abort = 0;
        dctx.abort_flag = &no_abort;
        if (*abort_flag == 0)
          ptx::mbar_wait(empty_bar + 8u * s, round & 1u, dctx, kSiteDrainLoads);
      }
    }
  }
}

template <int BN, int CtaGroup, typename AB, typename OutT>
__global__ void __launch_bounds__(EpiShape<BN>::kThreads, 1)
    gemm_sm100_kernel(const __grid_constant__ CUtensorMap tm_a,
                      const __grid_constant__ CUtensorMap tm_b,
                      const __grid_constant__ CUtensorMap tm_d,
                      const __grid_constant__ CUtensorMap tm_ws, const GemmParams p) {
#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ >= 1000)
  using L = GemmSmem<BN, CtaGroup>;
  using OT = OperandTraits<AB>;
  constexpr int kBK = OT::kBK;
  constexpr int kUmmaK = OT::kUmmaK;
  constexpr int kStoreCols = OutputTraits<OutT>::kStoreCols;
  constexpr uint32_t kIdesc = OT::kFp8 ? ptx::make_idesc_e4m3_f32(kBM * CtaGroup, L::kMmaN)
                                       : ptx::make_idesc_bf16_f32(kBM * CtaGroup, L::kMmaN);
  constexpr int kAccStages = L::kAccStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = ptx::smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw_addr);

  const int stages = p.ab_stages;
  const uint32_t epi_base = base + L::epi_offset(stages, p.reuse_ab);
  const uint32_t bar_base = base + L::barrier_offset(stages, p.epi_stages, p.reuse_ab);
  const uint32_t full_bar = bar_base;                       // [stages]
  const uint32_t empty_bar = bar_base + 8u * stages;        // [stages]
  const uint32_t tfull_bar = bar_base + 16u * stages;       // [2]
  const uint32_t tempty_bar = tfull_bar + 16u;              // [2]
  const uint32_t drain_bar = tempty_bar + 16u;              // [1]
  uint8_t* slot_ptr = base_ptr + (drain_bar + 8u - base);
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(slot_ptr);
  volatile int32_t* abort_flag = reinterpret_cast<volatile int32_t*>(slot_ptr + 4);

  const uint32_t warp = threadIdx.x >> 5;
  const uint32_t lane = ptx::lane_id();
  const uint32_t rank = (CtaGroup == 2) ? ptx::cluster_ctarank() : 0u;
  const bool leader = (CtaGroup == 1) || ((rank & 1u) == 0u);
  const uint32_t leader_rank = rank & ~1u;
  const uint16_t pair_mask = static_cast<uint16_t>(3u << leader_rank);  // both CTAs of the pair
  const int32_t cluster_ctas = p.sched.cluster_m * p.sched.cluster_n;
  DynArgs dyn;
  dyn.enabled = p.dynamic;
  dyn.layout = dyn_layout(base + L::dyn_offset(stages, p.epi_stages, p.reuse_ab));
  dyn.cluster_ctas = cluster_ctas;
  dyn.cluster_m = p.sched.cluster_m;
  dyn.rank = cluster_ctas > 1 ? ptx::cluster_ctarank() : 0u;
  // Cluster-wide barrier after the barrier initialisation and before exit: CTA pairs share
  // barriers and TMEM; the dynamic mode writes the other CTAs' work rings.
  const bool cluster_barriers = CtaGroup == 2 || (p.dynamic != 0 && cluster_ctas > 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      ptx::mbar_init(full_bar + 8u * s, 1);
      ptx::mbar_init(empty_bar + 8u * s, 1);
    }
    if (p.dynamic) {
      for (int i = 0; i < kWorkSlots; ++i) {
        ptx::mbar_init(dyn.layout.full + 8u * i, 1);
        ptx::mbar_init(dyn.layout.empty + 8u * i,
                       dyn_consumers(cluster_ctas, CtaGroup, EpiShape<BN>::kWarps));
      }
      ptx::mbar_init(dyn.layout.clc_bar, 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(tfull_bar + 8u * b, 1);
      ptx::mbar_init(tempty_bar + 8u * b, EpiShape<BN>::kWarps * CtaGroup);
    }
    ptx::mbar_init(drain_bar, 1);
    *abort_flag = 0;
    ptx::fence_mbarrier_init_cluster();
    ptx::fence_proxy_async_shared();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tensormap(&tm_a);
    ptx::prefetch_tensormap(&tm_b);
    ptx::prefetch_tensormap(&tm_d);
  }
  if (warp == 1) {
    ptx::tmem_alloc<CtaGroup>(ptx::smem_u32(const_cast<uint32_t*>(tmem_slot)), L::kTmemCols);
    ptx::tmem_relinquish<CtaGroup>();
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (cluster_barriers) ptx::cluster_sync();  // peer barriers initialised before use
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  ptx::WaitCtx ctx{abort_flag, p.status, p.timeout_ns};
  const SchedParams& sp = p.sched;
  const int k_iters = p.k_iters;

  using ES = EpiShape<BN>;
  // Each warpgroup changes its register budget inside its own role branch (512-wide tiles), so
  // the compiler allocates the producer / MMA code and the epilogue code separately.
  if (warp < static_cast<uint32_t>(ES::kFirstWarp)) {
  if constexpr (ES::kWide) ptx::setmaxnreg_dec<ES::kLowRegs>();
  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0 && (p.fault_inject & kInjectSkipLoads) == 0) {
      producer_loop<BN, CtaGroup, kBK, L::kStageBytes, L::kAStageBytes>(
          &tm_a, &tm_b, sp, k_iters, p.k_iters_per_split, stages, base, full_bar, empty_bar, rank,
          leader, ctx, p.l2_policy_a, p.l2_policy_b, p.stream_k, p.gated ? p.n : 0,
          p.num_splits, group_info(p), p.dp_tiles, dyn);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (leader && lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      SegmentIter si = make_segment_iter(sp, k_iters, p.k_iters_per_split, p.stream_k,
                                         p.num_splits, group_info(p), p.dp_tiles, p.dynamic);
      WorkReader reader(dyn.layout, dyn.rank);
      auto fetch = [&](Segment& out) -> bool {
        if (!dyn.enabled) return si.next(sp, out);
        int32_t cid;
        if (!reader.next(cid, ctx)) {
          ok = false;
          return false;
        }
        if (cid < 0) return false;
        si.it.cid = cid;
        return si.next(sp, out);
      };
      Segment sg;
      while (ok && fetch(sg)) {
        const int kb0 = sg.kb0, kb1 = sg.kb1;
        if (!ptx::mbar_wait(tempty_bar + 8u * acc, acc_phase ^ 1u, ctx, kSiteMmaTmemEmpty)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!ptx::mbar_wait(full_bar + 8u * stage, phase, ctx, kSiteMmaFull)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t sa = base + static_cast<uint32_t>(stage * L::kStageBytes);
          const uint32_t sb = sa + L::kAStageBytes;
          const uint64_t da = ptx::make_sw128_kmajor_desc(sa);
          const uint64_t db = ptx::make_sw128_kmajor_desc(sb);
#pragma unroll
          for (int k = 0; k < kBK / kUmmaK; ++k) {
            // Advance the start address by kUmmaK elements = 32 bytes inside the swizzled row;
            // MMA j reads B slot j (kBRowsPerMma rows further) into accumulator columns j * kMmaN.
#pragma unroll
            for (int j = 0; j < L::kNumMma; ++j) {
              const uint64_t dbj = db + static_cast<uint64_t>(2 * k + j * L::kBRowsPerMma * 8);
              const uint32_t dj = d_tmem + static_cast<uint32_t>(j * L::kMmaN);
              if constexpr (OT::kFp8) {
                ptx::umma_f8_ss<CtaGroup>(dj, da + static_cast<uint64_t>(2 * k), dbj, kIdesc,
                                          (kb > kb0 || k > 0) ? 1u : 0u);
              } else {
                ptx::umma_f16_ss<CtaGroup>(dj, da + static_cast<uint64_t>(2 * k), dbj, kIdesc,
                                           (kb > kb0 || k > 0) ? 1u : 0u);
              }
            }
          }
          const uint32_t eb = empty_bar + 8u * stage;
          if constexpr (CtaGroup == 1) {
            ptx::umma_commit<1>(eb);
          } else {
            ptx::umma_commit_pair(eb, pair_mask);
          }
          if (++stage == stages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        const uint32_t tb = tfull_bar + 8u * acc;
        if constexpr (CtaGroup == 1) {
          ptx::umma_commit<1>(tb);
        } else {
          ptx::umma_commit_pair(tb, pair_mask);
        }
        if (++acc == kAccStages) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // Drain: all MMAs issued by this thread complete before TMEM is freed.
      ptx::umma_commit<CtaGroup>(drain_bar);
      ptx::WaitCtx dctx{abort_flag, p.status, p.timeout_ns};
      volatile int32_t no_abort = 0;
      dctx.abort_flag = &no_abort;
      ptx::mbar_wait(drain_bar, 0u, dctx, kSiteDrainMma);
    }
    __syncwarp();
  }  // warps 2-3 of a 512-wide tile's first warpgroup have no role
  } else {
    if constexpr (ES::kWide) ptx::setmaxnreg_inc<ES::kHighRegs>();
    // ------------------------------------------------------------------ epilogue
    const uint32_t ew = warp - static_cast<uint32_t>(ES::kFirstWarp);  // 0 .. kWarps - 1
    const uint32_t quad = warp & 3u;  // TMEM lane quadrant this warp may access
    const uint32_t row_in_tile = quad * 32u;
    // The warp's share of the tile's columns: all of them, or (two warps per quadrant) half.
    const int half = static_cast<int>(ew) >> 2;
    int acc = 0;
    uint32_t acc_phase = 0;
    int epi_idx = 0;
    float alpha = p.alpha;
    if (p.scale_a != nullptr) alpha *= *p.scale_a;
    if (p.scale_b != nullptr) alpha *= *p.scale_b;
    const uint64_t pol_d = l2_policy(p.l2_policy_d);
    const bool has_bias = p.bias != nullptr;
    // 16-byte aligned bias: the epilogue reads whole chunks of it with vector loads.
    const bool bias_vec = has_bias && (reinterpret_cast<uintptr_t>(p.bias) & 15u) == 0;
    const bool has_src = p.src != nullptr;
    const bool gated = (BN == 512) && p.gated != 0;
    // Accumulator fully read into registers: hand the TMEM buffer back to the MMA warp.
    auto release_tmem = [&](int which) {
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        const uint32_t tb = tempty_bar + 8u * static_cast<uint32_t>(which);
        if constexpr (CtaGroup == 1) {
          ptx::mbar_arrive(tb);
        } else {
          ptx::mbar_arrive_cluster(ptx::mapa_shared(tb, leader_rank));
        }
      }
    };
    SegmentIter si = make_segment_iter(sp, p.k_iters, p.k_iters_per_split, p.stream_k,
                                       p.num_splits, group_info(p), p.dp_tiles, p.dynamic);
    // Dynamic mode: lane 0 reads the work ring and hands each entry to the warp.
    WorkReader reader(dyn.layout, dyn.rank);
    auto fetch = [&](Segment& out) -> bool {
      if (!dyn.enabled) return si.next(sp, out);
      int32_t cid = 0;
      int32_t got = 1;
      if (lane == 0) got = reader.next(cid, ctx) ? 1 : 0;
      cid = __shfl_sync(0xffffffffu, cid, 0);
      got = __shfl_sync(0xffffffffu, got, 0);
      if (!got || cid < 0) return false;
      si.it.cid = cid;
      return si.next(sp, out);
    };
    Segment sg;
    const int32_t cta_in_cluster = static_cast<int32_t>(ptx::cluster_ctaid_x()) +
                                   static_cast<int32_t>(ptx::cluster_ctaid_y()) * sp.cluster_m;
    while (fetch(sg)) {
      const int32_t pid_m = sg.pid_m, pid_n = sg.pid_n;
      // Split-K / Stream-K into D: only the segment holding a tile's first k-block adds the bias.
      const bool add_bias = has_bias && sg.kb0 == 0;
      // Stream-K with fixup, and split-K into peer memory: a segment with part of a tile's
      // k-blocks adds into the workspace.
      const bool partial = p.fixup != 0 && (sg.kb0 != 0 || sg.kb1 != p.k_iters);
      bool ok = ptx::mbar_wait(tfull_bar + 8u * acc, acc_phase, ctx, kSiteEpiTmemFull);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      ptx::tc_fence_after();
      if (p.tile_trace != nullptr && ew == 0 && lane == 0 && sg.index < p.trace_stride) {
        const int64_t cta = blockIdx.x + static_cast<int64_t>(gridDim.x) *
                                             (blockIdx.y + static_cast<int64_t>(gridDim.y) * blockIdx.z);
        int32_t* t = p.tile_trace + 2 * (cta * p.trace_stride + sg.index);
        t[0] = pid_m;
        t[1] = pid_n;
      }
      __syncwarp();
      const uint32_t t_row = tmem_base + (row_in_tile << 16) + static_cast<uint32_t>(acc * BN);
      const int32_t g_row = sg.row_base + pid_m * kBM + static_cast<int32_t>(row_in_tile);
      const int32_t my_row = g_row + static_cast<int32_t>(lane);
      // Rows of this warp that belong to the tile's problem (a grouped tile may end inside).
      const int32_t row_end = sg.row_end < p.m ? sg.row_end : p.m;
      // A gated 512-wide tile holds gate columns [0, 256) and up columns [256, 512) of the same
      // 256 output columns.
      const int out_cols = gated ? BN / 2 : BN;
      const int n_chunks = out_cols / kStoreCols;
      // This warp's chunks [c_begin, c_end) of the tile's columns.
      const int c_begin = half * n_chunks / ES::kHalves;
      const int c_end = (half + 1) * n_chunks / ES::kHalves;
      // This warp's 32 workspace rows (the CTA tile's workspace tile; partial segments only).
      // Stream-K numbers the split tiles after the data-parallel ones; split-K (L = K range)
      // shares one workspace tile between the K ranges of a tile.
      int32_t ws_cid = sg.cid - si.dp_tiles;
      if (partial && !p.stream_k) {
        int32_t l_idx;
        fast_divmod(sp.dm_clusters_per_problem, sg.cid, l_idx, ws_cid);
      }
      const int32_t ws_tile = partial ? ws_cid * cluster_ctas + cta_in_cluster : 0;
      const int32_t ws_row = ws_tile * kBM + static_cast<int32_t>(row_in_tile);
      // Reduce-scatter over peer memory: the rank owning this warp's rows (row blocks are whole
      // 128-row tiles, so all 32 rows have one owner; rows past M count for the last rank) and
      // the first of its rows in that rank's buffer.
      const bool rs = sizeof(OutT) == 4 && p.rs_ranks > 0;  // FP32 partial sums only
      int32_t rs_owner = 0;
      float* rs_rows = nullptr;
      if (rs) {
        rs_owner = p.rs_ranks - 1;
        for (int32_t q = 0; q < p.rs_ranks; ++q) {
          if (g_row < p.rs_row_start[q + 1]) {
            rs_owner = q;
            break;
          }
        }
        rs_rows = p.rs_dst[rs_owner] +
                  static_cast<int64_t>(g_row - p.rs_row_start[rs_owner]) * p.rs_ld;
      }

      // Stage 32 rows x 128 bytes of this warp's output (thread = row) in the next staging
      // buffer; returns the buffer's shared-memory address.
      auto stage = [&](const uint32_t (&words)[32]) -> uint32_t {
        const int buf = epi_idx % p.epi_stages;
        const uint32_t sbuf =
            epi_base + static_cast<uint32_t>((ew * p.epi_stages + buf) * kEpiBufBytes);
        if (lane == 0) epi_wait_buffer(p.epi_stages);
        __syncwarp();
        const uint32_t row_addr = sbuf + lane * 128u;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t chunk = static_cast<uint32_t>(j) ^ (lane & 7u);
          ptx::st_shared_v4(row_addr + (chunk << 4), words[4 * j], words[4 * j + 1],
                            words[4 * j + 2], words[4 * j + 3]);
        }
        ptx::fence_proxy_async_shared();
        __syncwarp();
        ++epi_idx;
        return sbuf;
      };
      // Round x (kStoreCols columns of this thread's row, from column col0) to D's type and
      // store it.
      auto store_chunk = [&](const float (&x)[kStoreCols], int32_t col0) {
        uint32_t packed[32];  // 128 bytes of this thread's output row
        if constexpr (sizeof(OutT) == 2) {
#pragma unroll
          for (int i = 0; i < 32; ++i) packed[i] = ptx::pack_bf16x2(x[2 * i], x[2 * i + 1]);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) packed[i] = __float_as_uint(x[i]);
        }
        const uint32_t sbuf = stage(packed);
        // The TMA box covers this warp's 32 rows and is clipped at D's last row; a grouped
        // tile whose group ends inside the box (before D ends) would write the next group's
        // rows with it, so there each thread stores its own row if it is in the group.
        // Boxes wholly outside D (the odd CTA of a pair past the last row tile) store nothing.
        const bool box = g_row + 32 <= row_end || (g_row < row_end && row_end == p.m);
        if (!box && g_row < row_end && col0 < p.n)
          store_row_chunk<OutT>(p, my_row, row_end, col0, packed);
        if (lane == 0) {
          if (box && col0 < p.n) {
            if (p.reduce_add) {
              ptx::tma_reduce_add_3d(&tm_d, sbuf, col0, g_row, sg.ab_batch);
            } else {
              ptx::tma_store_3d_hint(&tm_d, sbuf, col0, g_row, sg.ab_batch, pol_d);
            }
          }
          ptx::bulk_commit_group();
        }
        __syncwarp();
      };
      // Peer reduce-scatter: add x (kStoreCols FP32 columns of this thread's row) into the
      // owner's buffer, 32 columns (128 bytes) per staging buffer, copied out 4 rows x 128 bytes
      // per warp instruction (coalesced system-scope atomics).
      auto rs_add_chunk = [&](const float (&x)[kStoreCols], int32_t col0) {
#pragma unroll
        for (int sub = 0; sub < kStoreCols / 32; ++sub) {
          uint32_t words[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) words[i] = __float_as_uint(x[32 * sub + i]);
          const uint32_t sbuf = stage(words);
          const int32_t cbase = col0 + 32 * sub;
          const int32_t ch = static_cast<int32_t>(lane & 7u);
#pragma unroll
          for (int it = 0; it < 8; ++it) {
            const int32_t r = it * 4 + static_cast<int32_t>(lane >> 3);
            const int32_t col = cbase + 4 * ch;
            if (g_row + r < row_end && col < p.n) {
              const uint4 v = ptx::ld_shared_v4(
                  sbuf + static_cast<uint32_t>(r * 128 + ((ch ^ (r & 7)) << 4)));
              ptx::red_add_sys_v4(rs_rows + static_cast<int64_t>(r) * p.rs_ld + col, v);
            }
          }
          __syncwarp();
        }
      };
      // After this warp's last atomics of a tile: every lane's atomics before the warp's arrival
      // on the owner's count (system scope).
      auto rs_arrive = [&]() {
        ptx::fence_sc_sys();
        __syncwarp();
        if (lane == 0) ptx::red_release_sys_add_u32(p.rs_count[rs_owner], 1u);
      };
      auto add_bias_row = [&](float (&x)[kStoreCols], int32_t col0) {
        if (bias_vec && col0 + kStoreCols <= p.n) {
          // Every row needs the same kStoreCols values: all lanes load them with the same
          // 16-byte loads (one broadcast request each) and unpack the BF16 pairs.
          const __nv_bfloat16* bp = p.bias + col0;
#pragma unroll
          for (int q = 0; q < kStoreCols / 8; ++q) {
            const uint4 w = ptx::ld_global_nc_v4(bp + 8 * q);
            const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              x[8 * q + 2 * i] += __uint_as_float(ws[i] << 16);
              x[8 * q + 2 * i + 1] += __uint_as_float(ws[i] & 0xffff0000u);
            }
          }
          return;
        }
        // Otherwise lane l fetches bias[col0 + 32 h + l] (coalesced, bounds-checked) and the
        // values are broadcast across the warp with shuffles.
#pragma unroll
        for (int h = 0; h < kStoreCols / 32; ++h) {
          const int32_t n = col0 + 32 * h + static_cast<int32_t>(lane);
          const float bl = (n < p.n) ? __bfloat162float(p.bias[n]) : 0.f;
#pragma unroll
          for (int j = 0; j < 32; ++j) x[32 * h + j] += __shfl_sync(0xffffffffu, bl, j);
        }
      };

#pragma unroll 1
      for (int c = c_begin; c < c_end; ++c) {
        const int32_t col0 = pid_n * out_cols + c * kStoreCols;
        // C (beta * C source): this thread's 128-byte row chunk, fetched before the TMEM loads
        // so that the two latencies overlap.
        uint4 cs[8];
        if (has_src) load_row_chunk<OutT>(p, sg.ab_batch, my_row, col0, cs);
        float x[kStoreCols];
        if (!gated) {
          // kStoreCols accumulator columns of this thread's row (one 128-byte output row).
          uint32_t v[kStoreCols];
#pragma unroll
          for (int h = 0; h < kStoreCols / 32; ++h) {
            ptx::tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>(c * kStoreCols + 32 * h),
                                    *reinterpret_cast<uint32_t(*)[32]>(&v[32 * h]));
          }
          ptx::tmem_ld_wait();
          if (c == c_end - 1) release_tmem(acc);
#pragma unroll
          for (int j = 0; j < kStoreCols; ++j) x[j] = __uint_as_float(v[j]) * alpha;
        } else {
          // 32 gate and 32 up columns per TMEM round trip.
#pragma unroll
          for (int h = 0; h < kStoreCols / 32; ++h) {
            uint32_t vg[32], vu[32];
            const uint32_t tc = t_row + static_cast<uint32_t>(c * kStoreCols + 32 * h);
            ptx::tmem_ld_32x32b_x32(tc, vg);
            ptx::tmem_ld_32x32b_x32(tc + static_cast<uint32_t>(BN / 2), vu);
            ptx::tmem_ld_wait();
            if (c == c_end - 1 && h == kStoreCols / 32 - 1) release_tmem(acc);
            float gv[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) gv[j] = __uint_as_float(vg[j]) * alpha;
            act_inplace(p.act, gv);
#pragma unroll
            for (int j = 0; j < 32; ++j) x[32 * h + j] = gv[j] * (__uint_as_float(vu[j]) * alpha);
          }
        }
        if (partial) {
          // Add alpha * acc into the workspace, 32 FP32 columns (128 bytes) per TMA reduce.
#pragma unroll
          for (int sub = 0; sub < kStoreCols / 32; ++sub) {
            uint32_t words[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) words[i] = __float_as_uint(x[32 * sub + i]);
            const uint32_t sbuf = stage(words);
            if (lane == 0) {
              ptx::tma_reduce_add_3d(&tm_ws, sbuf, c * kStoreCols + 32 * sub, ws_row, 0);
              ptx::bulk_commit_group();
            }
            __syncwarp();
          }
          continue;
        }
        if (rs) {
          rs_add_chunk(x, col0);
          continue;
        }
        if (add_bias) add_bias_row(x, col0);
        if (has_src) add_row_chunk<OutT>(p.beta, cs, x);
        if (!gated) act_inplace(p.act, x);
        store_chunk(x, col0);
      }
      if (rs && !partial) rs_arrive();
      if (partial) {
        // Count this segment's k-blocks for its 32 rows; the warp that completes the count owns
        // every other segment's sum (their reduces completed before their counts were added).
        const int32_t cnt_idx = ws_tile * ES::kWarps + static_cast<int32_t>(ew);
        const int32_t mine = sg.kb1 - sg.kb0;
        int32_t last = 0;
        if (lane == 0) {
          ptx::bulk_wait_group<0>();
          ptx::fence_proxy_async_global();
          __threadfence();
          const int32_t before = atomicAdd(p.fixup_count + cnt_idx, mine);
          last = before + mine == p.k_iters ? 1 : 0;
          if (last) __threadfence();
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
          float* wrow = p.fixup_ws + static_cast<int64_t>(ws_row + static_cast<int32_t>(lane)) *
                                         p.ws_cols;
#pragma unroll 1
          for (int c = c_begin; c < c_end; ++c) {
            const int32_t col0 = pid_n * out_cols + c * kStoreCols;
            float x[kStoreCols];
            float* src = wrow + c * kStoreCols;
#pragma unroll
            for (int q = 0; q < kStoreCols / 4; ++q) {
              const uint4 v = ptx::ld_global_cg_v4(src + 4 * q);
              x[4 * q] = __uint_as_float(v.x);
              x[4 * q + 1] = __uint_as_float(v.y);
              x[4 * q + 2] = __uint_as_float(v.z);
              x[4 * q + 3] = __uint_as_float(v.w);
            }
            // Clear the workspace tile for the next launch.
#pragma unroll
            for (int q = 0; q < kStoreCols / 4; ++q) ptx::st_global_v4(src + 4 * q, 0u, 0u, 0u, 0u);
            if (rs) {
              rs_add_chunk(x, col0);  // the tile's sum crosses to its owner once
              continue;
            }
            if (has_bias) add_bias_row(x, col0);
            store_chunk(x, col0);
          }
          if (rs) rs_arrive();
          if (lane == 0) p.fixup_count[cnt_idx] = 0;
        }
      }
      if (++acc == kAccStages) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (lane == 0) ptx::bulk_wait_group<0>();
    __syncwarp();
  }

  // ------------------------------------------------------------------ teardown
  ptx::tc_fence_before();
  __syncthreads();
  if (cluster_barriers) ptx::cluster_sync();  // peers done with our barriers, TMEM and ring
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc<CtaGroup>(tmem_base, L::kTmemCols);
  }
#endif
}

// Small kernels that run the shared device code for host-side verification.
__global__ void sched_cluster_map_kernel(const SchedParams sp, int32_t* out, int64_t n) {
  int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i < n) {
    int32_t cm, cn;
    sched_map_cluster(sp, static_cast<int32_t>(i), cm, cn);
    out[2 * i] = cm;
    out[2 * i + 1] = cn;
  }
}

__global__ void fast_divmod_kernel(const FastDivmod f, const int32_t* x, int32_t* q, int32_t* r,
                                   int64_t n) {
  int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i < n) {
    int32_t qq, rr;
    fast_divmod(f, x[i], qq, rr);
    q[i] = qq;
    r[i] = rr;
  }
}

}  // namespace cpg
