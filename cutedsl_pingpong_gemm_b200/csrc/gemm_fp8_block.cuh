// Block-scaled FP8 E4M3 GEMM for sm_100a:
//   D[m, n] = alpha * sum_kb sa[kb][m] * sb[n / 128][kb] * (A[m, kb-block] . B[n, kb-block]^T)
// with 1 x 128 scales for A (one per row and 128-element k-block, stored k-block-major) and
// 128 x 128 scales for B (one per 128 x 128 block), fp32 scales (amax / 448), BF16 output.
//
// The tensor-core block-scaled MMA kinds take power-of-two (UE8M0 / UE4M3) scales on 16/32-wide
// k-blocks, which cannot represent fp32 scales, so the scaling is applied to fp32 partial sums:
//   warp 0     TMA producer (shared with the plain kernel), one 128-element k-block per stage.
//   warp 1     MMA issuer: each k-block's 4 tcgen05.mma kind::f8f6f4 write a fresh partial
//              product P_kb into one of 512 / BN TMEM partial buffers (128 lanes x BN fp32
//              columns), committed to that buffer's `part_full` barrier.
//   8 warps    promotion + epilogue: each thread owns BN / 2 columns of one row of the tile and
//              keeps those running fp32 sums in registers; per k-block it loads its part of P_kb
//              from TMEM, adds sa * sb * P_kb (packed fp32x2 FMAs), frees the partial buffer, and
//              after the last k-block rounds to BF16 and TMA-stores its 128-byte row chunks.
// Tiles are 128 x BN per CTA (256 x BN per CTA pair), BN = 128 or 256.  Per k-block a CTA loads
// 16 KiB of A and BN / CtaGroup rows of B from L2; the 256-wide tile does 1.5x the flops per
// loaded byte of the 128-wide one, whose throughput is bounded by that L2 -> SM traffic.  It has
// two partial buffers instead of four and 128 running sums per thread, which fit only after a
// register split: 384 threads launch with 168 registers each, then the warpgroup of the producer
// and MMA warps (two of its warps idle) drops to 40 and the two promotion warpgroups rise to 232
// (128 * 40 + 256 * 232 = 384 * 168).  Tile order, pairs, bounded waits and drains are as in
// gemm_sm100_kernel.
#pragma once
#include "gemm_kernel.cuh"

namespace cpg {

constexpr int kBlockEpiWarps = 8;

// Promotion warps: two per TMEM lane quadrant, each owning half of the tile's columns (warp w
// covers lanes 32 (w mod 4) .. +31 and columns (BN / 2) ((w - first) / 4) .. +BN/2-1), so a
// warp's columns never straddle a 128-column scale block of B.
template <int BN>
struct BlockShape {
  static_assert(BN == 128 || BN == 256, "block-scaled tiles are 128 or 256 columns wide");
  static constexpr int kParts = 512 / BN;                         // TMEM partial buffers
  static constexpr int kColsPerWarp = BN / (kBlockEpiWarps / 4);  // 64 or 128
  static constexpr bool kSplitRegs = BN == 256;
  static constexpr int kFirstPromoWarp = kSplitRegs ? 4 : 2;
  static constexpr int kThreads = (kFirstPromoWarp + kBlockEpiWarps) * 32;  // 320 or 384
  static constexpr int kLaunchRegs = 168;  // 65536 / 384, rounded down to a multiple of 8
  static constexpr int kLowRegs = 40;
  static constexpr int kHighRegs = 232;
  static_assert(!kSplitRegs || 128 * kLowRegs + 256 * kHighRegs == kThreads * kLaunchRegs,
                "register split must add up to the launch allocation");
};

template <int BN, int CtaGroup>
struct BlockSmem {
  static constexpr int kAStageBytes = kBM * kRowBytes;
  static constexpr int kBStageBytes = (BN / CtaGroup) * kRowBytes;
  static constexpr int kStageBytes = kAStageBytes + kBStageBytes;
  static constexpr int kTmemCols = 512;
  static __host__ __device__ int epi_offset(int stages) { return stages * kStageBytes; }
  static __host__ __device__ int barrier_offset(int stages, int epi_stages) {
    return epi_offset(stages) + kBlockEpiWarps * epi_stages * kEpiBufBytes;
  }
  // full[S], empty[S], part_full[P], part_empty[P], drain[1]; then tmem slot and abort flag;
  // then (16-byte aligned) the dynamic scheduler's kDynBytes (DynLayout).
  static __host__ __device__ int dyn_offset(int stages, int epi_stages) {
    return (barrier_offset(stages, epi_stages) + (2 * stages + 2 * BlockShape<BN>::kParts + 1) * 8 +
            16 + 15) & ~15;
  }
  static __host__ __device__ int bytes(int stages, int epi_stages, int /*reuse_ab*/) {
    int b = dyn_offset(stages, epi_stages) + kDynBytes + 1024;
    return b < kMinSmemForOneCtaPerSm ? kMinSmemForOneCtaPerSm : b;
  }
};

struct BlockScales {
  const float* sa;  // [ceil(K/128), M]
  const float* sb;  // [ceil(N/128), ceil(K/128)]
};

// acc[j] += s * v[j] for 32 columns (16 packed FMAs).
__device__ __forceinline__ void promote32(float* acc, float s, const uint32_t (&v)[32]) {
#pragma unroll
  for (int i = 0; i < 32; i += 2)
    ptx::fma2(acc[i], acc[i + 1], s, __uint_as_float(v[i]), __uint_as_float(v[i + 1]));
}

template <int BN, int CtaGroup>
__global__ void __launch_bounds__(BlockShape<BN>::kThreads, 1)
    gemm_fp8_block_kernel(const __grid_constant__ CUtensorMap tm_a,
                          const __grid_constant__ CUtensorMap tm_b,
                          const __grid_constant__ CUtensorMap tm_d, const GemmParams p,
                          const BlockScales scales) {
#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ >= 1000)
  using L = BlockSmem<BN, CtaGroup>;
  using Shape = BlockShape<BN>;
  constexpr int kParts = Shape::kParts;
  constexpr int kCols = Shape::kColsPerWarp;
  constexpr int kBK = OperandTraits<e4m3_t>::kBK;        // 128
  constexpr int kUmmaK = OperandTraits<e4m3_t>::kUmmaK;  // 32
  constexpr uint32_t kIdesc = ptx::make_idesc_e4m3_f32(kBM * CtaGroup, BN);

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = ptx::smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw_addr);

  const int stages = p.ab_stages;
  const uint32_t epi_base = base + L::epi_offset(stages);
  const uint32_t bar_base = base + L::barrier_offset(stages, p.epi_stages);
  const uint32_t full_bar = bar_base;
  const uint32_t empty_bar = bar_base + 8u * stages;
  const uint32_t pfull_bar = bar_base + 16u * stages;   // [kParts]
  const uint32_t pempty_bar = pfull_bar + 8u * kParts;  // [kParts]
  const uint32_t drain_bar = pempty_bar + 8u * kParts;
  uint8_t* slot_ptr = base_ptr + (drain_bar + 8u - base);
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(slot_ptr);
  volatile int32_t* abort_flag = reinterpret_cast<volatile int32_t*>(slot_ptr + 4);

  const uint32_t warp = threadIdx.x >> 5;
  const uint32_t lane = ptx::lane_id();
  const uint32_t rank = (CtaGroup == 2) ? ptx::cluster_ctarank() : 0u;
  const bool leader = (CtaGroup == 1) || ((rank & 1u) == 0u);
  const uint32_t leader_rank = rank & ~1u;
  const uint16_t pair_mask = static_cast<uint16_t>(3u << leader_rank);
  const int32_t cluster_ctas = p.sched.cluster_m * p.sched.cluster_n;
  DynArgs dyn;
  dyn.enabled = p.dynamic;
  dyn.layout = dyn_layout(base + L::dyn_offset(stages, p.epi_stages));
  dyn.cluster_ctas = cluster_ctas;
  dyn.cluster_m = p.sched.cluster_m;
  dyn.rank = cluster_ctas > 1 ? ptx::cluster_ctarank() : 0u;
  const bool cluster_barriers = CtaGroup == 2 || (p.dynamic != 0 && cluster_ctas > 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      ptx::mbar_init(full_bar + 8u * s, 1);
      ptx::mbar_init(empty_bar + 8u * s, 1);
    }
    for (int b = 0; b < kParts; ++b) {
      ptx::mbar_init(pfull_bar + 8u * b, 1);
      ptx::mbar_init(pempty_bar + 8u * b, kBlockEpiWarps * CtaGroup);
    }
    if (p.dynamic) {
      for (int i = 0; i < kWorkSlots; ++i) {
        ptx::mbar_init(dyn.layout.full + 8u * i, 1);
        ptx::mbar_init(dyn.layout.empty + 8u * i,
                       dyn_consumers(cluster_ctas, CtaGroup, kBlockEpiWarps));
      }
      ptx::mbar_init(dyn.layout.clc_bar, 1);
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
  if (cluster_barriers) ptx::cluster_sync();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  ptx::WaitCtx ctx{abort_flag, p.status, p.timeout_ns};
  const SchedParams& sp = p.sched;
  const int k_iters = p.k_iters;

  // Each warpgroup changes its register budget inside its own role branch, so the compiler
  // allocates the producer / MMA code and the promotion code separately.
  if (warp < static_cast<uint32_t>(Shape::kFirstPromoWarp)) {
    if constexpr (Shape::kSplitRegs) ptx::setmaxnreg_dec<Shape::kLowRegs>();
    if (warp == 0) {
      if (lane == 0 && (p.fault_inject & kInjectSkipLoads) == 0) {
        producer_loop<BN, CtaGroup, kBK, L::kStageBytes, L::kAStageBytes>(
            &tm_a, &tm_b, sp, k_iters, k_iters, stages, base, full_bar, empty_bar, rank, leader,
            ctx, p.l2_policy_a, p.l2_policy_b, 0, 0, 1, GroupInfo{0, nullptr, nullptr, 1}, 0,
            dyn);
      }
      __syncwarp();
    } else if (warp == 1) {
      if (leader && lane == 0) {
        int stage = 0;
        uint32_t phase = 0;
        int part = 0;
        uint32_t part_phase = 0;
        bool ok = true;
        TileSource tiles(sp, dyn);
        int32_t cid;
        while (ok && tiles.next(cid, ctx, ok, false)) {
          for (int kb = 0; kb < k_iters; ++kb) {
            if (!ptx::mbar_wait(pempty_bar + 8u * part, part_phase ^ 1u, ctx, kSiteMmaTmemEmpty) ||
                !ptx::mbar_wait(full_bar + 8u * stage, phase, ctx, kSiteMmaFull)) {
              ok = false;
              break;
            }
            ptx::tc_fence_after();
            const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(part * BN);
            const uint32_t sa = base + static_cast<uint32_t>(stage * L::kStageBytes);
            const uint64_t da = ptx::make_sw128_kmajor_desc(sa);
            const uint64_t db = ptx::make_sw128_kmajor_desc(sa + L::kAStageBytes);
#pragma unroll
            for (int k = 0; k < kBK / kUmmaK; ++k) {
              ptx::umma_f8_ss<CtaGroup>(d_tmem, da + static_cast<uint64_t>(2 * k),
                                        db + static_cast<uint64_t>(2 * k), kIdesc, k > 0 ? 1u : 0u);
            }
            const uint32_t eb = empty_bar + 8u * stage;
            const uint32_t pb = pfull_bar + 8u * part;
            if constexpr (CtaGroup == 1) {
              ptx::umma_commit<1>(eb);
              ptx::umma_commit<1>(pb);
            } else {
              ptx::umma_commit_pair(eb, pair_mask);
              ptx::umma_commit_pair(pb, pair_mask);
            }
            if (++stage == stages) {
              stage = 0;
              phase ^= 1u;
            }
            if (++part == kParts) {
              part = 0;
              part_phase ^= 1u;
            }
          }
        }
        ptx::umma_commit<CtaGroup>(drain_bar);
        ptx::WaitCtx dctx{abort_flag, p.status, p.timeout_ns};
        volatile int32_t no_abort = 0;
        dctx.abort_flag = &no_abort;
        ptx::mbar_wait(drain_bar, 0u, dctx, kSiteDrainMma);
      }
      __syncwarp();
    }
  } else {
    if constexpr (Shape::kSplitRegs) ptx::setmaxnreg_inc<Shape::kHighRegs>();
    // ---------------------------------------------------------------- promotion + epilogue
    const uint32_t ew = warp - Shape::kFirstPromoWarp;  // 0..7
    const uint32_t quad = warp & 3u;                    // TMEM lane quadrant this warp may access
    const uint32_t row_in_tile = quad * 32u;
    const uint32_t col_off = (ew >> 2) * kCols;
    const int64_t nkb_total = k_iters;
    const int32_t n_blocks = (p.n + 127) / 128;  // rows of sb
    int part = 0;
    uint32_t part_phase = 0;
    int epi_idx = 0;
    bool ok = true;
    TileSource tiles(sp, dyn);
    int32_t cid;
    int32_t executed = 0;
    for (; ok && tiles.next(cid, ctx, ok, true); ++executed) {
      int32_t pid_m, pid_n;
      work_tile_coords(sp, cid, pid_m, pid_n);
      if (p.tile_trace != nullptr && ew == 0 && lane == 0 && executed < p.trace_stride) {
        const int64_t cta = blockIdx.x + static_cast<int64_t>(gridDim.x) *
                                             (blockIdx.y + static_cast<int64_t>(gridDim.y) * blockIdx.z);
        int32_t* t = p.tile_trace + 2 * (cta * p.trace_stride + executed);
        t[0] = pid_m;
        t[1] = pid_n;
      }
      __syncwarp();
      const int32_t g_row = pid_m * kBM + static_cast<int32_t>(row_in_tile);
      const int32_t my_row = g_row + static_cast<int32_t>(lane);
      const bool row_ok = my_row < p.m;
      const int32_t col0 = pid_n * BN + static_cast<int32_t>(col_off);
      // This warp's columns lie in one 128-column scale block of B; past the last block of a
      // ragged N (the right half of a 256-wide edge tile) the scale reads are skipped.
      const int32_t nblk = col0 >> 7;
      const bool nblk_ok = nblk < n_blocks;
      const float* sb_row = scales.sb + static_cast<int64_t>(nblk_ok ? nblk : 0) * nkb_total;
      float acc[kCols];
#pragma unroll
      for (int j = 0; j < kCols; ++j) acc[j] = 0.f;
      // Scales are fetched kScalePrefetch k-blocks ahead into a register ring (the loop below
      // is unrolled by the ring length so the ring stays in registers): every k-block's scales
      // sit in a different cache line, and fetching them just in time stalls on memory latency.
      constexpr int kScalePrefetch = 4;
      float ring_a[kScalePrefetch], ring_b[kScalePrefetch];
#pragma unroll
      for (int j = 0; j < kScalePrefetch; ++j) {
        ring_a[j] = (j < k_iters && row_ok) ? scales.sa[static_cast<int64_t>(j) * p.m + my_row] : 0.f;
        ring_b[j] = (j < k_iters && nblk_ok) ? sb_row[j] : 0.f;
      }
      for (int kb0 = 0; ok && kb0 < k_iters; kb0 += kScalePrefetch) {
#pragma unroll
        for (int j = 0; j < kScalePrefetch; ++j) {
          const int kb = kb0 + j;
          if (!ok || kb >= k_iters) continue;
          const float s = ring_a[j] * ring_b[j];
          const int kn = kb + kScalePrefetch;
          ring_a[j] = (kn < k_iters && row_ok) ? scales.sa[static_cast<int64_t>(kn) * p.m + my_row]
                                               : 0.f;
          ring_b[j] = (kn < k_iters && nblk_ok) ? sb_row[kn] : 0.f;
          bool got = ptx::mbar_wait(pfull_bar + 8u * part, part_phase, ctx, kSiteEpiTmemFull);
          got = __all_sync(0xffffffffu, got);
          if (!got) {
            ok = false;
            continue;
          }
          ptx::tc_fence_after();
          const uint32_t t_row = tmem_base + (row_in_tile << 16) +
                                 static_cast<uint32_t>(part * BN) + col_off;
          const uint32_t pb = pempty_bar + 8u * static_cast<uint32_t>(part);
          auto release = [&]() {
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) {
              if constexpr (CtaGroup == 1) {
                ptx::mbar_arrive(pb);
              } else {
                ptx::mbar_arrive_cluster(ptx::mapa_shared(pb, leader_rank));
              }
            }
          };
          // Columns move through 64 registers, 32 per tcgen05.ld; the partial buffer is
          // released as soon as its last columns are in registers, before their FMAs.
          uint32_t va[32], vb[32];
          ptx::tmem_ld_32x32b_x32(t_row, va);
          ptx::tmem_ld_32x32b_x32(t_row + 32u, vb);
          ptx::tmem_ld_wait();
          if constexpr (kCols == 64) {
            release();
            promote32(acc, s, va);
            promote32(acc + 32, s, vb);
          } else {
            // The loads of columns 64-127 overlap the FMAs of columns 0-63.
            promote32(acc, s, va);
            ptx::tmem_ld_32x32b_x32(t_row + 64u, va);
            promote32(acc + 32, s, vb);
            ptx::tmem_ld_32x32b_x32(t_row + 96u, vb);
            ptx::tmem_ld_wait();
            release();
            promote32(acc + 64, s, va);
            promote32(acc + 96, s, vb);
          }
          if (++part == kParts) {
            part = 0;
            part_phase ^= 1u;
          }
        }
      }
      if (!ok) break;
      // Round this warp's columns of the row to BF16 and store them, one 128-byte row chunk
      // (64 columns) per TMA store.
      const bool has_bias = p.bias != nullptr;
#pragma unroll
      for (int c = 0; c < kCols; c += 64) {
        const int32_t cc = col0 + c;
        // Lane l holds bias[cc + l] and bias[cc + 32 + l]; shuffles broadcast them.
        const int32_t nb = cc + static_cast<int32_t>(lane);
        const float b0 = (has_bias && nb < p.n) ? __bfloat162float(p.bias[nb]) : 0.f;
        const float b1 = (has_bias && nb + 32 < p.n) ? __bfloat162float(p.bias[nb + 32]) : 0.f;
        uint32_t packed[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int j0 = 2 * i, j1 = 2 * i + 1;
          const float x0 =
              acc[c + j0] * p.alpha + __shfl_sync(0xffffffffu, j0 < 32 ? b0 : b1, j0 & 31);
          const float x1 =
              acc[c + j1] * p.alpha + __shfl_sync(0xffffffffu, j1 < 32 ? b0 : b1, j1 & 31);
          packed[i] = ptx::pack_bf16x2(x0, x1);
        }
        const int buf = epi_idx % p.epi_stages;
        const uint32_t sbuf =
            epi_base + static_cast<uint32_t>((ew * p.epi_stages + buf) * kEpiBufBytes);
        if (lane == 0) epi_wait_buffer(p.epi_stages);
        __syncwarp();
        const uint32_t row_addr = sbuf + lane * 128u;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t chunk = static_cast<uint32_t>(j) ^ (lane & 7u);
          ptx::st_shared_v4(row_addr + (chunk << 4), packed[4 * j], packed[4 * j + 1],
                            packed[4 * j + 2], packed[4 * j + 3]);
        }
        ptx::fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0) {
          if (g_row < p.m && cc < p.n) ptx::tma_store_3d(&tm_d, sbuf, cc, g_row, 0);
          ptx::bulk_commit_group();
        }
        __syncwarp();
        ++epi_idx;
      }
    }
    if (lane == 0) ptx::bulk_wait_group<0>();
    __syncwarp();
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (cluster_barriers) ptx::cluster_sync();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc<CtaGroup>(tmem_base, L::kTmemCols);
  }
#endif
}

}  // namespace cpg
