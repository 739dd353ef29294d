// Small-M ("decode") GEMM for sm_100a: D[M, N] = alpha * s_a * s_b * A[M, K] . B[N, K]^T + bias
// for M <= 128, the decode-like shapes where B (the weight, N x K) is read from HBM once and A
// holds a few token rows.
//
// The tile is transposed with respect to the plain kernel: the MMA computes D^T, B's rows on its
// M side (one TMEM lane each) and the M token rows of A on its N side (rounded up to 16; rows
// past M are zero-filled by TMA).  No 128-row A tile is padded out of a handful of rows, and every
// loaded byte of B feeds the tensor core once.  With so little math per byte, the MMA issue rate
// of a CTA's one issuing thread is one of its limits (about 100 cycles per tcgen05.mma whatever
// its N, plus about 200 per k-block for the barrier wait and the commit, measured with a clock64
// trace); the CTA-pair form (CG = 2) halves the MMA instructions per loaded byte: one
// tcgen05.mma.cta_group::2 with M = 256 covers 128 rows of B in each CTA of the pair, each CTA
// loading its own 128 rows of B and half of the token rows of A, the loads completing on the
// leader's barrier and the leader's commits releasing the stages of both CTAs.  Measured on
// B200 it ran level with or slower than single CTAs (CG = 1, 128-row tiles), the default.
//
// A tile of B (128 CG rows) alone leaves most SMs idle (N = 8192 gives 32 pair tiles), so the K
// range of a tile is split over S pairs (or CTAs) of one cluster (S = 1, 2 or 4; cluster dims
// (CG S, 1, 1), CTA rank CG kr + q for K range kr and position q in the pair; grid
// (CG S, ceil(N / (128 CG)))).  Each pair accumulates its K range in TMEM; the partial sums are
// then reduced through distributed shared memory, in one launch and without any global
// workspace: the 128 rows a CTA holds are dealt to the S CTAs holding the same rows in blocks
// of 128 / S rows.  Each CTA's receive slots have shared memory of their own, armed at start-up,
// so a CTA sends as soon as its own accumulators are complete: its warps holding another CTA's
// rows stage them in a send block (in its now free A/B stages) laid out as the owner's receive
// slot (rows padded by 16 bytes so a warp's 16-byte stores hit distinct banks), and one lane per
// 32 rows copies them to the owner with one bulk transfer (cp.async.bulk.shared::cluster)
// completing on the owner's receive barrier (plain per-thread remote stores of the same bytes
// measured ~10 us at M = 128; per-thread st.async into the owner's slot, the st_async option,
// level or slower).  The owner adds the S - 1 received blocks to its own rows, applies alpha,
// the FP8 scales and the bias, stages its rows of D^T as boxes of D (16 token rows x 32 columns)
// in its stages and writes each with one TMA store (128 two-byte global stores per thread
// measured ~6 us at M = 128).  Each launch is a programmatic dependent of the stream's previous
// kernel (the pdl option, see the prologue).
//
// Roles (320 threads): warp 0 TMA producer (one lane), warp 1 TMEM allocation and (leader CTA)
// MMA issuer (one lane), warps 2-9 the epilogue (warp w reads TMEM lane quadrant w mod 4, warps
// w and w + 4 splitting its columns).  Every wait is bounded (WaitCtx): on a timeout the status
// word records the site; in-flight TMA loads and MMAs are drained before the stages are reused
// or TMEM is freed, and the final cluster barrier keeps every CTA resident until every bulk copy
// into or out of its shared memory has completed.
#pragma once
#include "gemm_kernel.cuh"

namespace cpg {

constexpr int kDecodeThreads = 320;
constexpr int kDecodeEpiWarps = 8;   // two per TMEM lane quadrant, each with half the columns
constexpr int kDecodeMaxM = 128;      // MMA N: the token rows of one launch
constexpr int kDecodeTileN = 128;     // rows of B per CTA (the MMA's M per CTA, one TMEM lane each)
constexpr int kDecodeMaxSplits = 4;   // K ranges per cluster (owners of at least 32 rows each)
constexpr int kDecodeMaxStages = 12;
constexpr int32_t kSiteDecodeRecv = 11;  // the owner waiting for its peers' partial sums

struct DecodeParams {
  int32_t m, n, k;
  int32_t mma_n;       // round_up(M, 16)
  int32_t tmem_cols;   // power of two >= max(32, mma_n)
  int32_t k_iters;     // ceil(K / BK)
  int32_t kps;         // k-blocks per K range
  int32_t splits;      // K ranges per cluster: 1, 2 or 4
  int32_t stages;
  int32_t spin;        // producer / MMA lanes poll their barriers instead of sleeping
  int32_t rotate;      // start each tile's K range at a tile-dependent k-block (see below)
  int32_t pdl;         // launched as a programmatic dependent: set up, then wait (see below)
  int32_t st_async;    // partial sums sent by per-thread st.async instead of staged bulk copies
  float alpha;
  const float* scale_a;  // optional per-tensor FP8 scales (device scalars)
  const float* scale_b;
  const __nv_bfloat16* bias;  // optional, length N
  void* d;
  int64_t ldd;
  int32_t* status;
  uint64_t timeout_ns;
  int32_t l2_policy_a;  // 0 normal, 1 evict first, 2 evict last
  int32_t l2_policy_b;
};

// Shared-memory layout of one CTA (offsets from the 1024-byte aligned base), the same on host and
// device.  The send blocks of the reduction and the staging of D alias the A/B stages (used once
// this CTA's own loads and MMAs are done); the stages must hold epi_bytes().  The receive slots
// have memory of their own after the stages, so a peer may send while this CTA still computes.
struct DecodeLayout {
  uint32_t b_bytes;          // 128 rows of B x 128 bytes
  uint32_t stage_bytes;      // B rows + this CTA's mma_n / CG rows of A
  uint32_t row_floats;       // mma_n + 4 (16 bytes of padding per row)
  uint32_t block_bytes;      // one owner's rows of one sender: 128 / S rows
  uint32_t recv_bytes;       // (S - 1) blocks sent, and as many received
  uint32_t send_off;         // send blocks, at offset 0 of the stages
  uint32_t out_off;          // D boxes of the 4 TMEM lane quadrants, after the send blocks
  uint32_t recv_off;         // receive slots, after the stages
  uint32_t bar_off;          // full[stages], empty[stages], tmem_full, recv, drain
  uint32_t slot_off;         // TMEM base address, abort flag
  uint32_t bytes;            // dynamic shared memory to request (with the alignment slack)
  // One lane quadrant's box of D: mma_n token rows x 32 columns, unswizzled.
  __host__ __device__ uint32_t out_box_bytes(int out_elem_bytes) const {
    return (row_floats - 4u) * 32u * static_cast<uint32_t>(out_elem_bytes);
  }
  // Bytes of the stages the epilogue uses (send blocks and D boxes).
  __host__ __device__ uint32_t epi_bytes(int out_elem_bytes) const {
    return out_off + 4u * out_box_bytes(out_elem_bytes);
  }
};

__host__ __device__ inline DecodeLayout decode_layout(int stages, int mma_n, int splits,
                                                      int cta_group) {
  DecodeLayout l;
  l.b_bytes = kDecodeTileN * kRowBytes;
  l.stage_bytes = l.b_bytes + static_cast<uint32_t>(mma_n / cta_group) * kRowBytes;
  l.row_floats = static_cast<uint32_t>(mma_n) + 4u;
  l.block_bytes = static_cast<uint32_t>(kDecodeTileN / splits) * l.row_floats * 4u;
  l.recv_bytes = splits > 1 ? static_cast<uint32_t>(splits - 1) * l.block_bytes : 0u;
  l.send_off = 0u;
  l.out_off = (l.recv_bytes + 127u) & ~127u;
  l.recv_off = static_cast<uint32_t>(stages) * l.stage_bytes;
  l.bar_off = l.recv_off + ((l.recv_bytes + 127u) & ~127u);
  l.slot_off = l.bar_off + (2u * stages + 3u) * 8u;
  l.bytes = l.slot_off + 16u + 1024u;
  return l;
}

template <typename OutT>
__device__ __forceinline__ OutT to_out(float x);
template <>
__device__ __forceinline__ __nv_bfloat16 to_out<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
template <>
__device__ __forceinline__ float to_out<float>(float x) {
  return x;
}

template <typename AB, typename OutT, int CG>
__global__ void __launch_bounds__(kDecodeThreads, 1)
    gemm_decode_kernel(const __grid_constant__ CUtensorMap tm_a,
                       const __grid_constant__ CUtensorMap tm_b,
                       const __grid_constant__ CUtensorMap tm_d, const DecodeParams p) {
#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ >= 1000)
  using OT = OperandTraits<AB>;
  constexpr int kBK = OT::kBK;
  constexpr int kUmmaK = OT::kUmmaK;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = ptx::smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw_addr);

  const int stages = p.stages;
  const int S = p.splits;
  const DecodeLayout lay = decode_layout(stages, p.mma_n, S, CG);
  const uint32_t full_bar = base + lay.bar_off;
  const uint32_t empty_bar = full_bar + 8u * stages;
  const uint32_t tfull_bar = empty_bar + 8u * stages;
  const uint32_t recv_bar = tfull_bar + 8u;
  const uint32_t drain_bar = recv_bar + 8u;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(base_ptr + lay.slot_off);
  volatile int32_t* abort_flag = reinterpret_cast<volatile int32_t*>(base_ptr + lay.slot_off + 4);

  const uint32_t warp = threadIdx.x >> 5;
  const uint32_t lane = ptx::lane_id();
  const bool clustered = S * CG > 1;
  const uint32_t crank = clustered ? ptx::cluster_ctarank() : 0u;
  const uint32_t q = CG == 2 ? (crank & 1u) : 0u;              // position in the pair
  const uint32_t kr = CG == 2 ? (crank >> 1) : crank;          // K range of this CTA
  const bool leader = q == 0u;
  const uint32_t leader_rank = crank & ~1u;
  const uint16_t pair_mask = static_cast<uint16_t>(3u << leader_rank);
  const uint32_t rows_per_owner = static_cast<uint32_t>(kDecodeTileN / S);
  const int32_t n0 = static_cast<int32_t>(blockIdx.y) * (CG * kDecodeTileN) +
                     static_cast<int32_t>(q) * kDecodeTileN;  // this CTA's first row of B
  const int32_t a_row0 = static_cast<int32_t>(q) * (p.mma_n / CG);  // its first row of A
  const int32_t kb0 = static_cast<int32_t>(kr) * p.kps;
  const int32_t kb1 = min(p.k_iters, kb0 + p.kps);
  const bool has_k = kb1 > kb0;
  // All tiles stream the same k-block column of B at about the same time, and B's rows are K
  // elements apart, so the bytes in flight would share their offset modulo the row length and
  // crowd a few DRAM channels; starting each tile's walk over its K range at a different
  // k-block (rotate: tile * 5 modulo the range) spreads them.  Producer and MMA walk the same
  // order; the first k-block walked starts the accumulator.
  const int32_t nkb = kb1 > kb0 ? kb1 - kb0 : 1;
  const int32_t rot = p.rotate ? static_cast<int32_t>((blockIdx.y * 5u) % static_cast<uint32_t>(nkb)) : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      ptx::mbar_init(full_bar + 8u * s, 1);
      ptx::mbar_init(empty_bar + 8u * s, 1);
    }
    ptx::mbar_init(tfull_bar, 1);
    ptx::mbar_init(recv_bar, 1);
    ptx::mbar_init(drain_bar, 1);
    // The S - 1 blocks this CTA receives complete their bytes on recv_bar (armed before the
    // start-up cluster barrier, which every peer passes before it can send).
    if (S > 1)
      ptx::mbar_arrive_expect_tx(
          recv_bar, p.st_async ? static_cast<uint32_t>((S - 1) * rows_per_owner * p.mma_n * 4)
                               : lay.recv_bytes);
    *abort_flag = 0;
    ptx::fence_mbarrier_init_cluster();
    ptx::fence_proxy_async_shared();
  }
  // Programmatic dependent launch (pdl): the next kernel on the stream may be scheduled as soon as
  // every CTA of this one has started; this kernel in turn sets up (barriers, TMEM, the tensor
  // maps and an L2 prefetch of its first tiles of B, the weight) while the previous kernel
  // finishes, and waits for it to complete before any other global access (A, bias, scales, D,
  // the status word).  Without a programmatic dependency the wait returns at once.
  if (p.pdl) ptx::griddep_launch_dependents();
  const int32_t n_early = min(stages, kb1 - kb0);
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tensormap(&tm_a);
    ptx::prefetch_tensormap(&tm_b);
    ptx::prefetch_tensormap(&tm_d);
    if (p.pdl)
      for (int32_t i = 0; i < n_early; ++i)
        ptx::tma_prefetch_l2_3d(&tm_b, (kb0 + (i + rot) % nkb) * kBK, n0, 0);
  }
  if (warp == 1) {
    ptx::tmem_alloc<CG>(ptx::smem_u32(const_cast<uint32_t*>(tmem_slot)),
                        static_cast<uint32_t>(p.tmem_cols));
    ptx::tmem_relinquish<CG>();
  }
  ptx::griddep_wait();
  // Producer state (thread 0 = warp 0, lane 0).  A single CTA's loads complete on its own
  // barriers, which thread 0 has initialised: it fills the first `stages` stages (free by
  // construction) before the start-up barriers, whose latency then overlaps the first loads'
  // DRAM latency.  A pair's loads complete on the leader's barrier and wait for the cluster
  // barrier below.
  int p_stage = 0;
  uint32_t p_phase = 0;
  int32_t issued = 0;
  const uint64_t pol_a = l2_policy(p.l2_policy_a);
  const uint64_t pol_b = l2_policy(p.l2_policy_b);
  if constexpr (CG == 1) {
    if (threadIdx.x == 0) {
      for (; issued < n_early; ++issued) {
        const int32_t kb = kb0 + (issued + rot) % nkb;
        const uint32_t fb = full_bar + 8u * issued;
        const uint32_t sb = base + static_cast<uint32_t>(issued) * lay.stage_bytes;
        ptx::mbar_arrive_expect_tx(fb, lay.stage_bytes);
        ptx::tma_load_3d(&tm_b, sb, fb, kb * kBK, n0, 0, pol_b);
        ptx::tma_load_3d(&tm_a, sb + lay.b_bytes, fb, kb * kBK, a_row0, 0, pol_a);
      }
      p_stage = issued == stages ? 0 : issued;
      p_phase = issued == stages ? 1u : 0u;
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (clustered) ptx::cluster_sync();  // every CTA's barriers initialised before any remote use
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  ptx::WaitCtx ctx{abort_flag, p.status, p.timeout_ns};

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      int stage = p_stage;
      uint32_t phase = p_phase;
      for (int32_t i = issued; i < kb1 - kb0; ++i) {
        const int32_t kb = kb0 + (i + rot) % nkb;
        const uint32_t eb = empty_bar + 8u * stage;
        const bool slot_free = p.spin ? ptx::mbar_wait_spin(eb, phase ^ 1u, ctx, kSiteProducerEmpty)
                                      : ptx::mbar_wait(eb, phase ^ 1u, ctx, kSiteProducerEmpty);
        if (!slot_free) break;
        const uint32_t fb = full_bar + 8u * stage;
        const uint32_t sb = base + static_cast<uint32_t>(stage) * lay.stage_bytes;
        if constexpr (CG == 1) {
          ptx::mbar_arrive_expect_tx(fb, lay.stage_bytes);
          ptx::tma_load_3d(&tm_b, sb, fb, kb * kBK, n0, 0, pol_b);
          ptx::tma_load_3d(&tm_a, sb + lay.b_bytes, fb, kb * kBK, a_row0, 0, pol_a);
        } else {
          // Both CTAs' bytes complete on the leader's barrier.
          if (leader) ptx::mbar_arrive_expect_tx(fb, 2u * lay.stage_bytes);
          const uint32_t fb_leader = ptx::mapa_shared(fb, leader_rank);
          ptx::tma_load_3d_pair(&tm_b, sb, fb_leader, kb * kBK, n0, 0, pol_b);
          ptx::tma_load_3d_pair(&tm_a, sb + lay.b_bytes, fb_leader, kb * kBK, a_row0, 0, pol_a);
        }
        ++issued;
        if (++stage == stages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      // Drain: the last fill of every stage has landed before the stages are reused or the CTA
      // exits (bounded, and independent of an abort on the leader, whose full barriers count
      // both CTAs' bytes; the other CTA of a pair waits for its fills to be consumed).
      ptx::WaitCtx dctx = ctx;
      volatile int32_t no_abort = 0;
      dctx.abort_flag = &no_abort;
      for (int i = issued > stages ? issued - stages : 0; i < issued; ++i) {
        const uint32_t par = static_cast<uint32_t>((i / stages) & 1);
        if (leader)
          ptx::mbar_wait(full_bar + 8u * (i % stages), par, dctx, kSiteDrainLoads);
        else if (*abort_flag == 0)
          ptx::mbar_wait(empty_bar + 8u * (i % stages), par, dctx, kSiteDrainLoads);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer (leader)
    if (lane == 0 && leader) {
      const uint32_t idesc = OT::kFp8 ? ptx::make_idesc_e4m3_f32(CG * kDecodeTileN, p.mma_n)
                                      : ptx::make_idesc_bf16_f32(CG * kDecodeTileN, p.mma_n);
      // Descriptors as 32-bit low halves: stage s's B rows start at b_lo0 + s * stage_step,
      // its A rows at a_lo0 + s * stage_step.
      const uint32_t hi = ptx::sw128_desc_hi();
      const uint32_t stage_step = lay.stage_bytes >> 4;
      const uint32_t b_lo0 = ptx::sw128_desc_lo(base);
      const uint32_t a_lo0 = ptx::sw128_desc_lo(base + lay.b_bytes);
      uint32_t b_lo = b_lo0, a_lo = a_lo0;
      int stage = 0;
      uint32_t phase = 0;
      for (int32_t i = 0; i < kb1 - kb0; ++i) {
        const uint32_t fb = full_bar + 8u * stage;
        const bool full = p.spin ? ptx::mbar_wait_spin(fb, phase, ctx, kSiteMmaFull)
                                 : ptx::mbar_wait(fb, phase, ctx, kSiteMmaFull);
        if (!full) break;
        // The stage's bytes arrived through the async proxy (TMA) and are read through it (the
        // MMA): the completed barrier phase orders them; no tcgen05 fence is needed here.
#pragma unroll
        for (int k = 0; k < kBK / kUmmaK; ++k)
          ptx::umma_ss_lohi<CG, OT::kFp8>(tmem_base, b_lo + 2u * k, a_lo + 2u * k, hi, idesc,
                                          (i > 0 || k > 0) ? 1u : 0u);
        if constexpr (CG == 1) {
          ptx::umma_commit<1>(empty_bar + 8u * stage);
        } else {
          ptx::umma_commit_pair(empty_bar + 8u * stage, pair_mask);
        }
        if (++stage == stages) {
          stage = 0;
          phase ^= 1u;
          b_lo = b_lo0;
          a_lo = a_lo0;
        } else {
          b_lo += stage_step;
          a_lo += stage_step;
        }
      }
      if constexpr (CG == 1) {
        ptx::umma_commit<1>(tfull_bar);
      } else {
        ptx::umma_commit_pair(tfull_bar, pair_mask);
      }
      // No MMA may still read the stages or write TMEM when they are reused or freed.
      ptx::umma_commit<CG>(drain_bar);
      ptx::WaitCtx dctx = ctx;
      volatile int32_t no_abort = 0;
      dctx.abort_flag = &no_abort;
      ptx::mbar_wait(drain_bar, 0u, dctx, kSiteDrainMma);
    }
    __syncwarp();
  }
  // ---------------------------------------------------------------- reduction + epilogue
  // The epilogue warps wait for the accumulators; warps 0 and 1 reach the barrier below after
  // draining their loads and MMAs, so past it this CTA's stages are free for the send blocks and
  // the D boxes.  The receive slots have memory of their own, armed at start-up: a peer sends as
  // soon as its own accumulators are complete, with no cluster-wide barrier in between.
  bool ok = true;
  if (warp >= 2) {
    ok = ptx::mbar_wait(tfull_bar, 0u, ctx, kSiteEpiTmemFull);
    ok = __all_sync(0xffffffffu, ok) && *abort_flag == 0;
    ptx::tc_fence_after();
  }
  ptx::fence_proxy_async_shared();  // the stages' async-proxy use ends before generic stores
  __syncthreads();
  // The closing cluster barrier is split: each warp arrives once it has no more business with a
  // peer's shared memory (warps 0 and 1 now, a sender once its copy is issued, an owner once its
  // partial sums have arrived), and all wait at the very end, so no CTA leaves while a bulk copy
  // may still read or write its shared memory, and the wait is mostly over by then.
  if (clustered && warp < 2) ptx::cluster_arrive();
  if (warp >= 2) {
    // Warp w reads TMEM lane quadrant w mod 4 (rows 32 quad .. 32 quad + 31 of this CTA's tile)
    // and the 16-column chunks c = half + 2 j of the accumulator (token rows 16 c .. 16 c + 15).
    const uint32_t quad = warp & 3u;
    const uint32_t half = (warp - 2u) >> 2;
    const int chunks = p.mma_n / 16;
    const uint32_t row = quad * 32u + lane;
    const uint32_t owner = (quad * 32u) / rows_per_owner;  // K range owning these rows
    const uint32_t local = row - owner * rows_per_owner;  // row within the owner's block
    const uint32_t t_row = tmem_base + ((quad * 32u) << 16);
    const bool read_tmem = ok && has_k;
    uint32_t v[4][16];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = static_cast<int>(half) + 2 * j;
      if (read_tmem && c < chunks) ptx::tmem_ld_32x32b_x16(t_row + static_cast<uint32_t>(16 * c), v[j]);
    }
    if (read_tmem) {
      ptx::tmem_ld_wait();
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int i = 0; i < 16; ++i) v[j][i] = 0u;
    }
    if (owner != kr) {
      // Stage these rows' partial sums in the send block for their owner (laid out as the
      // owner's receive slot: 128 / S rows of mma_n + 4 floats); once both warps of the quadrant
      // are done, one lane copies its 32 rows to the owner in one bulk transfer, completing the
      // bytes on the owner's receive barrier.
      const uint32_t block = owner < kr ? owner : owner - 1u;
      const uint32_t slot = kr < owner ? kr : kr - 1u;  // this CTA's slot at the owner
      const uint32_t dst_rank = owner * CG + q;
      const uint32_t q_off = (quad * 32u - owner * rows_per_owner) * lay.row_floats * 4u;
      if (p.st_async) {
        // Each lane stores its row's partial sums straight into the owner's receive slot, 16
        // bytes per st.async, each completing on the owner's receive barrier.
        const uint32_t rdst = ptx::mapa_shared(
            base + lay.recv_off + slot * lay.block_bytes + q_off + lane * lay.row_floats * 4u,
            dst_rank);
        const uint32_t rbar = ptx::mapa_shared(recv_bar, dst_rank);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int c = static_cast<int>(half) + 2 * j;
          if (c < chunks) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
              ptx::st_async_v4(rdst + static_cast<uint32_t>(64 * c + 16 * i), v[j][4 * i],
                               v[j][4 * i + 1], v[j][4 * i + 2], v[j][4 * i + 3], rbar);
          }
        }
      } else {
        const uint32_t src = base + lay.send_off + block * lay.block_bytes + q_off;
        const uint32_t dst = src + lane * lay.row_floats * 4u;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int c = static_cast<int>(half) + 2 * j;
          if (c < chunks) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
              ptx::st_shared_v4(dst + static_cast<uint32_t>(64 * c + 16 * i), v[j][4 * i],
                                v[j][4 * i + 1], v[j][4 * i + 2], v[j][4 * i + 3]);
          }
        }
        ptx::fence_proxy_async_shared();  // generic stores before the bulk copy reads them
        ptx::named_barrier_sync(1u + quad, 64u);
        if (half == 0u && lane == 0u)
          ptx::bulk_copy_to_cluster(
              ptx::mapa_shared(base + lay.recv_off + slot * lay.block_bytes + q_off, dst_rank),
              src, 32u * lay.row_floats * 4u, ptx::mapa_shared(recv_bar, dst_rank));
      }
      __syncwarp();
      if (clustered) ptx::cluster_arrive();
    } else {
      bool got = S == 1 || ptx::mbar_wait(recv_bar, 0u, ctx, kSiteDecodeRecv);
      got = __all_sync(0xffffffffu, got) && ok;
      if (clustered) ptx::cluster_arrive();
      if (got) {
        const int32_t n = n0 + static_cast<int32_t>(row);
        float scale = p.alpha;
        if (p.scale_a != nullptr) scale *= *p.scale_a;
        if (p.scale_b != nullptr) scale *= *p.scale_b;
        const float bias = (p.bias != nullptr && n < p.n) ? __bfloat162float(p.bias[n]) : 0.f;
        // The quadrant's box of D (mma_n token rows x its 32 columns, unswizzled): lane l holds
        // column l of every row, so each row of the box is one conflict-free warp store; each
        // chunk of 16 rows is written by one TMA store (rows past M, columns past N clipped).
        const uint32_t box_off = lay.out_off + quad * lay.out_box_bytes(sizeof(OutT));
        OutT* box = reinterpret_cast<OutT*>(base_ptr + box_off);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int c = static_cast<int>(half) + 2 * j;
          if (c < chunks) {
            float acc[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) acc[i] = __uint_as_float(v[j][i]);
            for (int sidx = 0; sidx < S - 1; ++sidx) {
              const uint32_t r_addr =
                  base + lay.recv_off +
                  ((static_cast<uint32_t>(sidx) * rows_per_owner + local) * lay.row_floats +
                   static_cast<uint32_t>(16 * c)) * 4u;
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const uint4 w = ptx::ld_shared_v4(r_addr + 16u * i);
                acc[4 * i] += __uint_as_float(w.x);
                acc[4 * i + 1] += __uint_as_float(w.y);
                acc[4 * i + 2] += __uint_as_float(w.z);
                acc[4 * i + 3] += __uint_as_float(w.w);
              }
            }
#pragma unroll
            for (int i = 0; i < 16; ++i)
              box[(16 * c + i) * 32 + static_cast<int>(lane)] = to_out<OutT>(acc[i] * scale + bias);
          }
        }
        ptx::fence_proxy_async_shared();  // the box's generic stores before the TMA stores
        __syncwarp();
        const int32_t col0 = n0 + static_cast<int32_t>(quad * 32u);
        if (lane == 0 && col0 < p.n) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int c = static_cast<int>(half) + 2 * j;
            if (c < chunks)
              ptx::tma_store_3d(&tm_d, base + box_off + static_cast<uint32_t>(c * 16 * 32) *
                                                            static_cast<uint32_t>(sizeof(OutT)),
                                col0, 16 * c, 0);
          }
          ptx::bulk_commit_group();
          ptx::bulk_wait_group_read<0>();  // the box is read before its memory is released
        }
        __syncwarp();
      }
    }
  }

  if (clustered) ptx::cluster_wait();  // no CTA leaves while a peer may still copy into or out of it
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc<CG>(tmem_base, static_cast<uint32_t>(p.tmem_cols));
  }
#endif
}

}  // namespace cpg
