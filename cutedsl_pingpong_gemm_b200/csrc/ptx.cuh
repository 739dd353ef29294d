// Inline-PTX wrappers for sm_100a: mbarriers, TMA (tensor bulk copies), tcgen05 (TMEM alloc,
// UMMA issue/commit, TMEM loads) and cluster helpers.  Every wait here is bounded: the caller
// passes a WaitCtx and gets `false` back when the deadline passed or another role aborted.
#pragma once
#include <cuda.h>
#include <stdint.h>

namespace cpg {
namespace ptx {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint32_t lane_id() { return threadIdx.x & 31u; }

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- cluster special registers
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t clusterid_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t clusterid_y() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.y;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t nclusterid_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_ctaid_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctaid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_ctaid_y() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctaid.y;" : "=r"(r));
  return r;
}

// Address of the same shared-memory offset in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_sync() {
  cluster_arrive();
  cluster_wait();
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbarrier_init_cluster() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Arrive on a barrier that may live in another CTA of the cluster (address from mapa_shared).
// Default (CTA-scope) semantics: the barriers here order tensor-memory accesses, which the
// tcgen05 fences around the arrive / wait already cover, so no cluster-scope fence is needed.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// As mbar_try_wait, but the thread may be suspended for up to `suspend_ns` nanoseconds while the
// phase is incomplete (it resumes as soon as the phase completes), so waiting warps sleep
// instead of spinning.
__device__ __forceinline__ bool mbar_try_wait_suspend(uint32_t bar, uint32_t parity,
                                                      uint32_t suspend_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(suspend_ns)
      : "memory");
  return ok != 0;
}

// Shared state for bounded waits: a deadline and a CTA-wide abort flag in shared memory.
struct WaitCtx {
  volatile int32_t* abort_flag;  // shared memory; nonzero once any role gave up
  int32_t* status;               // global error word (first error wins), may be null
  uint64_t timeout_ns;
};

// Error codes written to the device status word.  The low byte names the wait site.
enum : int32_t {
  kStatusOk = 0,
  kStatusTimeoutBase = 0x100,
};

__device__ __noinline__ void record_timeout(const WaitCtx& ctx, int32_t site) {
  *ctx.abort_flag = 1;
  if (ctx.status != nullptr) atomicCAS(ctx.status, 0, kStatusTimeoutBase | site);
}

// Wait until the phase with parity `parity` of barrier `bar` completed.  Returns false when the
// deadline passes (recording `site`) or when another role already aborted.  Between checks of
// the deadline and the abort flag the thread sleeps in try_wait for at most kWaitSuspendNs.
constexpr uint32_t kWaitSuspendNs = 1000000;  // 1 ms

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, const WaitCtx& ctx,
                                          int32_t site) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    if (mbar_try_wait_suspend(bar, parity, kWaitSuspendNs)) return true;
    if (*ctx.abort_flag) return false;
    if (globaltimer() - t0 > ctx.timeout_ns) {
      record_timeout(ctx, site);
      return false;
    }
  }
}

// Non-blocking test of the phase with parity `parity`.
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// As mbar_wait, but polling with the non-blocking test_wait instead of sleeping in try_wait: for
// loops whose work per phase is short next to a suspended thread's wake-up (the small-M
// kernel's producer and MMA lanes).  Bounded the same way (deadline and abort flag, checked
// every 256 polls).
__device__ __forceinline__ bool mbar_wait_spin(uint32_t bar, uint32_t parity, const WaitCtx& ctx,
                                               int32_t site) {
  if (mbar_test_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    for (int i = 0; i < 256; ++i)
      if (mbar_test_wait(bar, parity)) return true;
    if (*ctx.abort_flag) return false;
    if (globaltimer() - t0 > ctx.timeout_ns) {
      record_timeout(ctx, site);
      return false;
    }
  }
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

// Tensor maps are 3-D: (columns, rows, batch); an unbatched operand has one batch (z = 0).

// Tiled load into this CTA's shared memory, completing its bytes on barrier `bar` (this CTA).
// Prefetch a tile of a tensor into L2 (no shared memory, no barrier).  Only a hint: L2 is the
// coherence point, so a prefetch never makes a later load see stale data.
__device__ __forceinline__ void tma_prefetch_l2_3d(const CUtensorMap* m, int32_t x, int32_t y,
                                                   int32_t z) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global [%0, {%1, %2, %3}];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(x), "r"(y), "r"(z)
               : "memory");
}

// Programmatic dependent launch: let the grid launched after this one on the stream be scheduled
// once every CTA of this grid has executed this (or exited) ...
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
// ... and, in that later grid, wait until the grids it depends on have completed and their memory
// operations are visible (returns at once without such a dependency).
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ void tma_load_3d(const CUtensorMap* m, uint32_t dst, uint32_t bar,
                                            int32_t x, int32_t y, int32_t z, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar), "r"(x), "r"(y), "r"(z), "l"(policy)
      : "memory");
}

// Tiled load for a CTA pair: data lands in this CTA's shared memory, the transaction bytes
// complete on `cluster_bar`, which may be the pair leader's barrier (address from mapa_shared).
__device__ __forceinline__ void tma_load_3d_pair(const CUtensorMap* m, uint32_t dst,
                                                 uint32_t cluster_bar, int32_t x, int32_t y,
                                                 int32_t z, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(cluster_bar), "r"(x), "r"(y), "r"(z), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_store_3d(const CUtensorMap* m, uint32_t src, int32_t x,
                                             int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(m)),
      "r"(src), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// As tma_store_3d, with an L2 eviction-priority policy for the written lines.
__device__ __forceinline__ void tma_store_3d_hint(const CUtensorMap* m, uint32_t src, int32_t x,
                                                  int32_t y, int32_t z, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%2, %3, %4}], "
      "[%1], %5;" ::"l"(reinterpret_cast<uint64_t>(m)),
      "r"(src), "r"(x), "r"(y), "r"(z), "l"(policy)
      : "memory");
}

// Element-wise add of a shared-memory box into global memory (fp32 split-K accumulation in L2).
__device__ __forceinline__ void tma_reduce_add_3d(const CUtensorMap* m, uint32_t src, int32_t x,
                                                  int32_t y, int32_t z) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.bulk_group [%0, {%2, %3, %4}], "
      "[%1];" ::"l"(reinterpret_cast<uint64_t>(m)),
      "r"(src), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ uint32_t clusterid_z() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.z;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t nclusterid_y() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.y;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait_group() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// L2 eviction-priority policies for TMA loads.
__device__ __forceinline__ uint64_t policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---------------------------------------------------------------- tcgen05: TMEM allocation
template <int CtaGroup>
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  if constexpr (CtaGroup == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                 "r"(ncols)
                 : "memory");
  } else {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                 "r"(ncols)
                 : "memory");
  }
}

template <int CtaGroup>
__device__ __forceinline__ void tmem_relinquish() {
  if constexpr (CtaGroup == 1) {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  } else {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
}

template <int CtaGroup>
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  if constexpr (CtaGroup == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
  } else {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
  }
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---------------------------------------------------------------- tcgen05: UMMA
// Shared-memory matrix descriptor (tcgen05 "matrix descriptor"):
//   [0,14)  start address >> 4      [16,30) leading byte offset >> 4
//   [32,46) stride byte offset >> 4 [46,48) version = 1
//   [49,52) base offset             [52]    LBO mode
//   [61,64) layout: 0 none, 2 = 128B swizzle, 4 = 64B, 6 = 32B
// For K-major operands staged by TMA with 128-byte swizzle, rows are 128 bytes, 8-row core
// groups are 1024 bytes apart (SBO = 1024) and LBO is unused (encoded as 1).
__device__ __forceinline__ uint64_t make_sw128_kmajor_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;              // LBO (unused for swizzled K-major)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;      // SBO = 1024 bytes
  d |= static_cast<uint64_t>(1u) << 46;              // version
  d |= static_cast<uint64_t>(2u) << 61;              // SWIZZLE_128B
  return d;
}

// Instruction descriptor for kind::f16 with BF16 A/B, F32 accumulate, both K-major.
__host__ __device__ constexpr uint32_t make_idesc_bf16_f32(int M, int N) {
  return (1u << 4)                                   // c_format = F32
         | (1u << 7)                                 // a_format = BF16
         | (1u << 10)                                // b_format = BF16
         | (0u << 15) | (0u << 16)                   // A, B K-major
         | (static_cast<uint32_t>(N >> 3) << 17)     // N >> 3
         | (static_cast<uint32_t>(M >> 4) << 24);    // M >> 4
}

// Instruction descriptor for kind::f8f6f4 with E4M3 A/B, F32 accumulate, both K-major.
__host__ __device__ constexpr uint32_t make_idesc_e4m3_f32(int M, int N) {
  return (1u << 4)                                   // c_format = F32
         | (0u << 7)                                 // a_format = E4M3
         | (0u << 10)                                // b_format = E4M3
         | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread.
template <int CtaGroup>
__device__ __forceinline__ void umma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  if constexpr (CtaGroup == 1) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}

template <int CtaGroup>
__device__ __forceinline__ void umma_f8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
  if constexpr (CtaGroup == 1) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}

// Matrix descriptors split into their two 32-bit halves: only the low half (start address >> 4
// and the unused LBO field) depends on the address, so a k-step or a stage advance is one 32-bit
// add, and the 64-bit descriptor is packed inside the MMA instruction's asm.
__device__ __forceinline__ uint32_t sw128_desc_lo(uint32_t smem_addr) {
  return ((smem_addr >> 4) & 0x3FFFu) | (1u << 16);
}
__host__ __device__ constexpr uint32_t sw128_desc_hi() {
  return (1024u >> 4) | (1u << (46 - 32)) | (2u << (61 - 32));
}

template <int CtaGroup, bool Fp8>
__device__ __forceinline__ void umma_ss_lohi(uint32_t d_tmem, uint32_t a_lo, uint32_t b_lo,
                                             uint32_t hi, uint32_t idesc, uint32_t accumulate) {
  if constexpr (CtaGroup == 1 && !Fp8) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t.reg .b64 da, db;\n\t"
        "setp.ne.b32 p, %5, 0;\n\t"
        "mov.b64 da, {%1, %3};\n\t"
        "mov.b64 db, {%2, %3};\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %4, p;\n\t}" ::"r"(d_tmem),
        "r"(a_lo), "r"(b_lo), "r"(hi), "r"(idesc), "r"(accumulate)
        : "memory");
  } else if constexpr (CtaGroup == 1 && Fp8) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t.reg .b64 da, db;\n\t"
        "setp.ne.b32 p, %5, 0;\n\t"
        "mov.b64 da, {%1, %3};\n\t"
        "mov.b64 db, {%2, %3};\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], da, db, %4, p;\n\t}" ::"r"(d_tmem),
        "r"(a_lo), "r"(b_lo), "r"(hi), "r"(idesc), "r"(accumulate)
        : "memory");
  } else if constexpr (!Fp8) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t.reg .b64 da, db;\n\t"
        "setp.ne.b32 p, %5, 0;\n\t"
        "mov.b64 da, {%1, %3};\n\t"
        "mov.b64 db, {%2, %3};\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], da, db, %4, p;\n\t}" ::"r"(d_tmem),
        "r"(a_lo), "r"(b_lo), "r"(hi), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t.reg .b64 da, db;\n\t"
        "setp.ne.b32 p, %5, 0;\n\t"
        "mov.b64 da, {%1, %3};\n\t"
        "mov.b64 db, {%2, %3};\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], da, db, %4, p;\n\t}" ::"r"(d_tmem),
        "r"(a_lo), "r"(b_lo), "r"(hi), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}

// Arrive once on `bar` when all previously issued tcgen05 async operations of this thread
// complete.  `bar` is a shared::cluster address (own CTA or, for pairs, the peer CTA).
template <int CtaGroup>
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  if constexpr (CtaGroup == 1) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     bar)
                 : "memory");
  } else {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     bar)
                 : "memory");
  }
}

// CTA-pair form: arrive once on the barrier at offset `bar` in every CTA of `cta_mask` (the two
// CTAs of the pair) when the pair MMAs issued by this thread complete.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(bar),
      "h"(cta_mask)
      : "memory");
}

// ---------------------------------------------------------------- tcgen05: TMEM -> registers
// 32 lanes x 32 consecutive 32-bit columns: thread t receives lane (quadrant*32 + t).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 32 lanes x 16 consecutive 32-bit columns: thread t receives lane (quadrant*32 + t).
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------- misc
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %2, %1;" : "=r"(r) : "f"(lo), "f"(hi));
  return r;
}

// (c0, c1) += s * (x0, x1): one packed fp32x2 FMA (round-to-nearest per element, the same result
// as two fmaf calls), which halves the FMA issue slots on sm_100a.
__device__ __forceinline__ void fma2(float& c0, float& c1, float s, float x0, float x1) {
  asm("{\n\t.reg .b64 xa, sa, ca;\n\t"
      "mov.b64 xa, {%2, %3};\n\t"
      "mov.b64 sa, {%4, %4};\n\t"
      "mov.b64 ca, {%0, %1};\n\t"
      "fma.rn.f32x2 ca, xa, sa, ca;\n\t"
      "mov.b64 {%0, %1}, ca;\n\t}"
      : "+f"(c0), "+f"(c1)
      : "f"(x0), "f"(x1), "f"(s));
}

// Per-warpgroup register budget changes (all four warps of a warpgroup execute the same one).
template <int N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

// 16-byte read-only global load (the address must be 16-byte aligned).
__device__ __forceinline__ uint4 ld_global_nc_v4(const void* ptr) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(ptr));
  return r;
}

// 16-byte global load cached in L2 only (data other SMs wrote during this kernel).
__device__ __forceinline__ uint4 ld_global_cg_v4(const void* ptr) {
  uint4 r;
  asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(ptr)
               : "memory");
  return r;
}

// Orders this thread's completed async-proxy (TMA) global writes before its later generic
// accesses, e.g. the release of a flag other CTAs acquire.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// 16-byte global store (the address must be 16-byte aligned).
__device__ __forceinline__ void st_global_v4(void* ptr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.global.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(ptr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

// ---------------------------------------------------------------- cluster launch control
// Ask to cancel the launch of a cluster of this grid that has not started yet.  The 16-byte
// response is written (async proxy) to this CTA's shared memory at `resp` and completes 16 bytes
// of transaction on `bar`.  After a response reported failure no further request may be issued.
__device__ __forceinline__ void clc_try_cancel(uint32_t resp, uint32_t bar) {
  asm volatile(
      "clusterlaunchcontrol.try_cancel.async.shared::cta.mbarrier::complete_tx::bytes.b128 "
      "[%0], [%1];" ::"r"(resp),
      "r"(bar)
      : "memory");
}

// Decode the response at `resp`: the x index of the cancelled cluster's first CTA, or -1 when
// the request failed (no cluster left to cancel).
__device__ __forceinline__ int32_t clc_query_first_x(uint32_t resp) {
  uint64_t lo, hi;
  asm volatile("ld.shared.v2.b64 {%0, %1}, [%2];" : "=l"(lo), "=l"(hi) : "r"(resp) : "memory");
  uint32_t ok, x;
  asm volatile(
      "{\n\t.reg .b128 r;\n\t.reg .pred p;\n\t"
      "mov.b128 r, {%2, %3};\n\t"
      "clusterlaunchcontrol.query_cancel.is_canceled.pred.b128 p, r;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t"
      "mov.u32 %1, 0;\n\t"
      "@p clusterlaunchcontrol.query_cancel.get_first_ctaid::x.b32.b128 %1, r;\n\t}"
      : "=r"(ok), "=r"(x)
      : "l"(lo), "l"(hi));
  return ok ? static_cast<int32_t>(x) : -1;
}

// Store / arrive on another CTA's shared memory (addresses from mapa_shared) with cluster-scope
// release, and wait with cluster-scope acquire: for data handed between the CTAs of a cluster.
__device__ __forceinline__ void st_shared_cluster_u32(uint32_t cluster_addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}
__device__ __forceinline__ void st_shared_cluster_v4(uint32_t cluster_addr, uint32_t a,
                                                     uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared::cluster.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(cluster_addr), "r"(a),
               "r"(b), "r"(c), "r"(d)
               : "memory");
}
// Bulk copy of `bytes` (a multiple of 16, both addresses 16-byte aligned) from this CTA's shared
// memory into another CTA's of the cluster (addresses from mapa_shared), completing the bytes
// on that CTA's barrier `cluster_bar`.
__device__ __forceinline__ void bulk_copy_to_cluster(uint32_t dst_cluster, uint32_t src,
                                                     uint32_t bytes, uint32_t cluster_bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, "
      "[%3];" ::"r"(dst_cluster),
      "r"(src), "r"(bytes), "r"(cluster_bar)
      : "memory");
}
// Named barrier `id` over `threads` threads (a multiple of 32) of this CTA.
// Asynchronous 16-byte store into a cluster peer's shared memory, completing its bytes on the
// peer's mbarrier (both addresses from mapa_shared).
__device__ __forceinline__ void st_async_v4(uint32_t cluster_addr, uint32_t a, uint32_t b,
                                            uint32_t c, uint32_t d, uint32_t cluster_bar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];"
      ::"r"(cluster_addr), "r"(a), "r"(b), "r"(c), "r"(d), "r"(cluster_bar)
      : "memory");
}

__device__ __forceinline__ void named_barrier_sync(uint32_t id, uint32_t threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ uint32_t ld_shared_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ void mbar_arrive_release_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_acquire_cluster(uint32_t bar, uint32_t parity,
                                                              uint32_t suspend_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(suspend_ns)
      : "memory");
  return ok != 0;
}
// Bounded like mbar_wait, with cluster-scope acquire.
__device__ __forceinline__ bool mbar_wait_acquire_cluster(uint32_t bar, uint32_t parity,
                                                          const WaitCtx& ctx, int32_t site) {
  const uint64_t t0 = globaltimer();
  while (true) {
    if (mbar_try_wait_acquire_cluster(bar, parity, kWaitSuspendNs)) return true;
    if (*ctx.abort_flag) return false;
    if (globaltimer() - t0 > ctx.timeout_ns) {
      record_timeout(ctx, site);
      return false;
    }
  }
}

// ---------------------------------------------------------------- peer memory (NVLink)
// 16-byte atomic add to global memory that may live on another GPU (a peer allocation mapped
// into this process), atomic with respect to every GPU of the system.
__device__ __forceinline__ void red_add_sys_v4(float* ptr, const uint4& v) {
  asm volatile("red.relaxed.sys.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(ptr),
               "f"(__uint_as_float(v.x)), "f"(__uint_as_float(v.y)), "f"(__uint_as_float(v.z)),
               "f"(__uint_as_float(v.w))
               : "memory");
}
__device__ __forceinline__ void red_release_sys_add_u32(uint32_t* ptr, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* ptr) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(ptr) : "memory");
  return v;
}
__device__ __forceinline__ void fence_sc_sys() { asm volatile("fence.sc.sys;" ::: "memory"); }
__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

}  // namespace ptx
}  // namespace cpg
