// Small-M ("decode") GEMM for sm_100a: D[M, N] = alpha * s_a * s_b * A[M, K] . B[N, K]^T + bias
// for M <= 128, the decode-like shapes where B (the weight, N x K) is read from HBM once and A
// holds a few token rows.
//
// The tile is transposed with respect to the plain kernel: each CTA computes D^T for 128 R rows
// of B (R = 1 or 2 row blocks, one M = 128 MMA and one TMEM accumulator each), so B's rows fill
// the MMA's M side (128 TMEM lanes per block) and the M token rows of A are the MMA's N (rounded
// up to 16; rows past M are zero-filled by TMA).  No 128-row A tile is padded out of a handful of
// rows, and every loaded byte of B feeds the tensor core once.  Two row blocks per CTA halve the
// re-reads of A from L2 (every tile reads all of A), which matter once A has 64 rows or more.
//
// A tile of B alone leaves most SMs idle (N = 8192 gives 64 or 32 tiles), so the K range of a
// tile is split over the S CTAs of a cluster (S = 1, 2 or 4; cluster dims (S, 1, 1), grid
// (S, ceil(N / (128 R)))).  Each CTA accumulates its K range in TMEM; the partial sums are then
// reduced through distributed shared memory, in one launch and without any global workspace:
// the 128 R rows of the tile are dealt to the CTAs in blocks of 128 R / S rows (CTA r owns rows
// [r 128 R / S, (r + 1) 128 R / S)).  Once every CTA of the cluster has finished its MMAs and its
// loads (a cluster barrier), the A/B stages are free and serve as receive buffers: the warps
// holding another CTA's rows store them there (st.shared::cluster, 16-byte vectors, rows padded
// by 16 bytes so a warp's stores hit distinct banks) and arrive on that CTA's receive barrier
// with cluster-scope release; the owner adds the S - 1 received rows to its own, applies alpha,
// the FP8 scales and the bias and writes its rows of D^T as columns of D (for each token row m, a
// warp writes 32 consecutive elements).
//
// Roles (192 threads): warp 0 TMA producer (one lane), warp 1 TMEM allocation and MMA issuer
// (one lane), warps 2-5 the epilogue (warp w reads TMEM lane quadrant w mod 4 of every block).
// Every wait is bounded (WaitCtx): on a timeout the status word records the site; in-flight TMA
// loads and MMAs are drained before the stages are reused or TMEM is freed, and the final
// cluster barrier keeps every CTA resident until no peer can still write into its shared memory.
#pragma once
#include "gemm_kernel.cuh"

namespace cpg {

constexpr int kDecodeThreads = 192;
constexpr int kDecodeMaxM = 128;      // MMA N: the token rows of one launch
constexpr int kDecodeTileN = 128;     // rows of B per row block (the MMA's M, one TMEM lane each)
constexpr int kDecodeMaxBlocks = 2;   // row blocks per CTA
constexpr int kDecodeMaxSplits = 4;   // CTAs per cluster (owners of at least 32 rows each)
constexpr int kDecodeMaxStages = 12;
constexpr int32_t kSiteDecodeRecv = 11;  // the owner waiting for its peers' partial sums

struct DecodeParams {
  int32_t m, n, k;
  int32_t mma_n;       // round_up(M, 16)
  int32_t tmem_cols;   // power of two >= max(32, mma_n)
  int32_t k_iters;     // ceil(K / BK)
  int32_t kps;         // k-blocks per CTA of a cluster
  int32_t splits;      // CTAs per cluster: 1, 2 or 4
  int32_t rblocks;     // 128-row blocks of B per CTA: 1 or 2
  int32_t stages;
  int32_t spin;        // producer / MMA lanes poll their barriers instead of sleeping
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

// Shared-memory layout (offsets from the 1024-byte aligned base), the same on host and device.
// The receive buffer of the reduction aliases the A/B stages (used only after every CTA of the
// cluster has finished with them).
struct DecodeLayout {
  uint32_t b_bytes;          // 128 R rows of B x 128 bytes
  uint32_t stage_bytes;      // B rows + mma_n rows of A
  uint32_t recv_row_floats;  // mma_n + 4 (16 bytes of padding per row)
  uint32_t recv_bytes;       // (S - 1) * 128 R / S rows
  uint32_t bar_off;          // full[stages], empty[stages], tmem_full, recv, drain
  uint32_t slot_off;         // TMEM base address, abort flag
  uint32_t bytes;            // dynamic shared memory to request (with the alignment slack)
};

__host__ __device__ inline DecodeLayout decode_layout(int stages, int mma_n, int splits,
                                                      int rblocks) {
  DecodeLayout l;
  l.b_bytes = static_cast<uint32_t>(rblocks) * kDecodeTileN * kRowBytes;
  l.stage_bytes = l.b_bytes + static_cast<uint32_t>(mma_n) * kRowBytes;
  l.recv_row_floats = static_cast<uint32_t>(mma_n) + 4u;
  const uint32_t recv_rows =
      splits > 1 ? (splits - 1) * (static_cast<uint32_t>(rblocks) * kDecodeTileN / splits) : 0u;
  l.recv_bytes = recv_rows * l.recv_row_floats * 4u;
  l.bar_off = static_cast<uint32_t>(stages) * l.stage_bytes;
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

template <typename AB, typename OutT>
__global__ void __launch_bounds__(kDecodeThreads, 1)
    gemm_decode_kernel(const __grid_constant__ CUtensorMap tm_a,
                       const __grid_constant__ CUtensorMap tm_b, const DecodeParams p) {
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
  const int R = p.rblocks;
  const DecodeLayout lay = decode_layout(stages, p.mma_n, S, R);
  const uint32_t full_bar = base + lay.bar_off;
  const uint32_t empty_bar = full_bar + 8u * stages;
  const uint32_t tfull_bar = empty_bar + 8u * stages;
  const uint32_t recv_bar = tfull_bar + 8u;
  const uint32_t drain_bar = recv_bar + 8u;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(base_ptr + lay.slot_off);
  volatile int32_t* abort_flag = reinterpret_cast<volatile int32_t*>(base_ptr + lay.slot_off + 4);

  const uint32_t warp = threadIdx.x >> 5;
  const uint32_t lane = ptx::lane_id();
  const uint32_t rank = S > 1 ? ptx::cluster_ctarank() : 0u;
  const uint32_t rows_per_owner = static_cast<uint32_t>(R * kDecodeTileN / S);
  const int32_t n0 = static_cast<int32_t>(blockIdx.y) * R * kDecodeTileN;
  const int32_t kb0 = static_cast<int32_t>(rank) * p.kps;
  const int32_t kb1 = min(p.k_iters, kb0 + p.kps);
  const bool has_k = kb1 > kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      ptx::mbar_init(full_bar + 8u * s, 1);
      ptx::mbar_init(empty_bar + 8u * s, 1);
    }
    ptx::mbar_init(tfull_bar, 1);
    ptx::mbar_init(recv_bar, S > 1 ? (S - 1) * rows_per_owner : 1u);
    ptx::mbar_init(drain_bar, 1);
    *abort_flag = 0;
    ptx::fence_mbarrier_init_cluster();
    ptx::fence_proxy_async_shared();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tensormap(&tm_a);
    ptx::prefetch_tensormap(&tm_b);
  }
  if (warp == 1) {
    ptx::tmem_alloc<1>(ptx::smem_u32(const_cast<uint32_t*>(tmem_slot)),
                       static_cast<uint32_t>(p.tmem_cols));
    ptx::tmem_relinquish<1>();
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (S > 1) ptx::cluster_sync();  // every CTA's receive barrier initialised before any arrive
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  ptx::WaitCtx ctx{abort_flag, p.status, p.timeout_ns};

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      const uint64_t pol_a = l2_policy(p.l2_policy_a);
      const uint64_t pol_b = l2_policy(p.l2_policy_b);
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      for (int32_t kb = kb0; kb < kb1; ++kb) {
        const bool slot_free = p.spin ? ptx::mbar_wait_spin(empty_bar + 8u * stage, phase ^ 1u, ctx,
                                                       kSiteProducerEmpty)
                                 : ptx::mbar_wait(empty_bar + 8u * stage, phase ^ 1u, ctx,
                                                  kSiteProducerEmpty);
        if (!slot_free) break;
        const uint32_t fb = full_bar + 8u * stage;
        const uint32_t sb = base + static_cast<uint32_t>(stage) * lay.stage_bytes;
        ptx::mbar_arrive_expect_tx(fb, lay.stage_bytes);
        ptx::tma_load_3d(&tm_b, sb, fb, kb * kBK, n0, 0, pol_b);
        ptx::tma_load_3d(&tm_a, sb + lay.b_bytes, fb, kb * kBK, 0, 0, pol_a);
        ++issued;
        if (++stage == stages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      // Drain: the last fill of every stage has landed before the CTA may exit (bounded, and
      // independent of an abort: a TMA write must not reach freed shared memory).
      ptx::WaitCtx dctx = ctx;
      volatile int32_t no_abort = 0;
      dctx.abort_flag = &no_abort;
      for (int i = issued > stages ? issued - stages : 0; i < issued; ++i)
        ptx::mbar_wait(full_bar + 8u * (i % stages), static_cast<uint32_t>((i / stages) & 1),
                       dctx, kSiteDrainLoads);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = OT::kFp8 ? ptx::make_idesc_e4m3_f32(kDecodeTileN, p.mma_n)
                                      : ptx::make_idesc_bf16_f32(kDecodeTileN, p.mma_n);
      // Descriptors as 32-bit low halves: stage s's B block r starts at
      // b_lo0 + s * stage_step + r * block_step, its A rows a_lo0 + s * stage_step.
      const uint32_t hi = ptx::sw128_desc_hi();
      const uint32_t stage_step = lay.stage_bytes >> 4;
      const uint32_t block_step = (kDecodeTileN * kRowBytes) >> 4;
      const uint32_t b_lo0 = ptx::sw128_desc_lo(base);
      const uint32_t a_lo0 = ptx::sw128_desc_lo(base + lay.b_bytes);
      uint32_t b_lo = b_lo0, a_lo = a_lo0;
      int stage = 0;
      uint32_t phase = 0;
      for (int32_t kb = kb0; kb < kb1; ++kb) {
        const bool full = p.spin ? ptx::mbar_wait_spin(full_bar + 8u * stage, phase, ctx, kSiteMmaFull)
                                 : ptx::mbar_wait(full_bar + 8u * stage, phase, ctx, kSiteMmaFull);
        if (!full) break;
        // The stage's bytes arrived through the async proxy (TMA) and are read through it (the
        // MMA): the completed barrier phase orders them; no tcgen05 fence is needed here.
#pragma unroll
        for (int k = 0; k < kBK / kUmmaK; ++k) {
          const uint32_t acc = (kb > kb0 || k > 0) ? 1u : 0u;
          for (int r = 0; r < R; ++r)
            ptx::umma_ss_lohi<1, OT::kFp8>(tmem_base + static_cast<uint32_t>(r * p.mma_n),
                                           b_lo + r * block_step + 2u * k, a_lo + 2u * k, hi,
                                           idesc, acc);
        }
        ptx::umma_commit<1>(empty_bar + 8u * stage);
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
      ptx::umma_commit<1>(tfull_bar);
      // No MMA may still write TMEM when it is freed.
      ptx::umma_commit<1>(drain_bar);
      ptx::WaitCtx dctx = ctx;
      volatile int32_t no_abort = 0;
      dctx.abort_flag = &no_abort;
      ptx::mbar_wait(drain_bar, 0u, dctx, kSiteDrainMma);
    }
    __syncwarp();
  }
  // Every CTA of the cluster has drained its loads and MMAs (warps 0 and 1 above) and its
  // epilogue warps have seen the accumulators complete: the stages of all of them are free to
  // receive partial sums.
  bool ok = true;
  if (warp >= 2) {
    ok = ptx::mbar_wait(tfull_bar, 0u, ctx, kSiteEpiTmemFull);
    ok = __all_sync(0xffffffffu, ok) && *abort_flag == 0;
    ptx::tc_fence_after();
  }
  ptx::fence_proxy_async_shared();  // the stages' async-proxy use ends before generic stores
  if (S > 1) ptx::cluster_sync();
  if (warp >= 2) {
    // ---------------------------------------------------------------- reduction + epilogue
    const uint32_t quad = warp & 3u;
    const int chunks = p.mma_n / 16;
    const bool read_tmem = ok && has_k;
    // Sends first (they never wait), then the owned rows (which wait for the peers' sends).
    for (int r = 0; r < R; ++r) {
      const uint32_t row = static_cast<uint32_t>(r * kDecodeTileN) + quad * 32u + lane;
      const uint32_t owner = (row - lane) / rows_per_owner;  // uniform over the warp
      if (owner == rank) continue;
      const uint32_t t_row = tmem_base + ((quad * 32u) << 16) + static_cast<uint32_t>(r * p.mma_n);
      const uint32_t slot = rank < owner ? rank : rank - 1u;
      const uint32_t local = row - owner * rows_per_owner;
      const uint32_t dst = ptx::mapa_shared(
          base + (slot * rows_per_owner + local) * lay.recv_row_floats * 4u, owner);
      for (int c = 0; c < chunks; ++c) {
        uint32_t v[16];
        if (read_tmem) {
          ptx::tmem_ld_32x32b_x16(t_row + static_cast<uint32_t>(16 * c), v);
          ptx::tmem_ld_wait();
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = 0u;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j)
          ptx::st_shared_cluster_v4(dst + static_cast<uint32_t>(64 * c + 16 * j), v[4 * j],
                                    v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
      }
      ptx::mbar_arrive_release_cluster(ptx::mapa_shared(recv_bar, owner));
    }
    bool waited = false, got = ok;
    for (int r = 0; r < R; ++r) {
      const uint32_t row = static_cast<uint32_t>(r * kDecodeTileN) + quad * 32u + lane;
      const uint32_t owner = (row - lane) / rows_per_owner;
      if (owner != rank) continue;
      if (!waited && S > 1) {
        bool g = ptx::mbar_wait_acquire_cluster(recv_bar, 0u, ctx, kSiteDecodeRecv);
        got = __all_sync(0xffffffffu, g) && ok;
        waited = true;
      }
      if (!got) break;
      const uint32_t t_row = tmem_base + ((quad * 32u) << 16) + static_cast<uint32_t>(r * p.mma_n);
      const int32_t n = n0 + static_cast<int32_t>(row);
      float scale = p.alpha;
      if (p.scale_a != nullptr) scale *= *p.scale_a;
      if (p.scale_b != nullptr) scale *= *p.scale_b;
      const bool n_ok = n < p.n;
      const float bias = (p.bias != nullptr && n_ok) ? __bfloat162float(p.bias[n]) : 0.f;
      const uint32_t local = row - rank * rows_per_owner;
      OutT* d = static_cast<OutT*>(p.d);
      for (int c = 0; c < chunks; ++c) {
        uint32_t v[16];
        if (has_k) {
          ptx::tmem_ld_32x32b_x16(t_row + static_cast<uint32_t>(16 * c), v);
          ptx::tmem_ld_wait();
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = 0u;
        }
        float acc[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[j] = __uint_as_float(v[j]);
        for (int src = 0; src < S - 1; ++src) {
          const uint32_t r_addr = base + ((static_cast<uint32_t>(src) * rows_per_owner + local) *
                                              lay.recv_row_floats +
                                          static_cast<uint32_t>(16 * c)) *
                                             4u;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint4 w = ptx::ld_shared_v4(r_addr + 16u * j);
            acc[4 * j] += __uint_as_float(w.x);
            acc[4 * j + 1] += __uint_as_float(w.y);
            acc[4 * j + 2] += __uint_as_float(w.z);
            acc[4 * j + 3] += __uint_as_float(w.w);
          }
        }
        if (n_ok) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int32_t m = 16 * c + j;
            if (m < p.m)
              d[static_cast<int64_t>(m) * p.ldd + n] = to_out<OutT>(acc[j] * scale + bias);
          }
        }
      }
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (S > 1) ptx::cluster_sync();  // no CTA leaves while a peer may still store into it
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc<1>(tmem_base, static_cast<uint32_t>(p.tmem_cols));
  }
#endif
}

}  // namespace cpg
