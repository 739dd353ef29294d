// Owner side of the split-K reduce-scatter over peer memory.
//
// Every rank's GEMM (gemm_sm100_kernel with rs_ranks > 0) adds its FP32 partial tiles straight
// into the buffer of the rank that owns their rows, with system-scope atomics over NVLink, and
// each epilogue warp then raises the owner's arrival counter with a release add.  The owner runs
// peer_finish_kernel on its own stream after its GEMM: it waits until the counter has reached the
// number of arrivals all ranks make on its rows (cumulative over calls, so the counter is never
// reset), rounds its rows to BF16 (+ bias) and clears the buffer for the call after next (the
// caller alternates two buffers, so a rank that runs ahead adds into the other one).
#pragma once
#include <cuda_bf16.h>
#include <stdint.h>

#include "gemm_kernel.cuh"
#include "ptx.cuh"

namespace cpg {

// Thread 0 of each CTA waits (bounded by timeout_ns, or until another CTA gave up); on a timeout
// it records kStatusTimeoutBase | kSitePeerArrivals in *status and the CTA writes nothing.
// Rows are 4-column aligned (cols % 4 == 0, ldw % 4 == 0, ldd % 4 == 0).
__global__ void peer_finish_kernel(float* __restrict__ w, int64_t ldw, const uint32_t* count,
                                   uint32_t target, int64_t rows, int64_t cols,
                                   __nv_bfloat16* __restrict__ d, int64_t ldd,
                                   const __nv_bfloat16* __restrict__ bias, int32_t* status,
                                   uint64_t timeout_ns) {
  __shared__ int32_t go;
  if (threadIdx.x == 0) {
    int32_t ok = 1;
    const uint64_t t0 = ptx::globaltimer();
    // Compared modulo 2^32: the counter only grows, by the arrivals of one call at a time.
    while (static_cast<int32_t>(ptx::ld_acquire_sys_u32(count) - target) < 0) {
      if (*reinterpret_cast<volatile int32_t*>(status) != 0 ||
          ptx::globaltimer() - t0 > timeout_ns) {
        atomicCAS(status, 0, ptx::kStatusTimeoutBase | kSitePeerArrivals);
        ok = 0;
        break;
      }
      __nanosleep(256);
    }
    go = ok;
  }
  __syncthreads();
  if (!go) return;
  const int64_t vcols = cols / 4;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    float* wr = w + r * ldw;
    __nv_bfloat16* dr = d + r * ldd;
    for (int64_t c = threadIdx.x; c < vcols; c += blockDim.x) {
      // L2 loads (not L1): the atomics of the other GPUs were performed in this GPU's L2.
      const uint4 v = ptx::ld_global_cg_v4(wr + 4 * c);
      float x[4] = {__uint_as_float(v.x), __uint_as_float(v.y), __uint_as_float(v.z),
                    __uint_as_float(v.w)};
      if (bias != nullptr) {
#pragma unroll
        for (int j = 0; j < 4; ++j) x[j] += __bfloat162float(bias[4 * c + j]);
      }
      uint2 packed;
      packed.x = ptx::pack_bf16x2(x[0], x[1]);
      packed.y = ptx::pack_bf16x2(x[2], x[3]);
      *reinterpret_cast<uint2*>(dr + 4 * c) = packed;
      *reinterpret_cast<uint4*>(wr + 4 * c) = make_uint4(0u, 0u, 0u, 0u);
    }
  }
}

}  // namespace cpg
