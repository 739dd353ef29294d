// FP8 E4M3 quantisation and FP32 -> BF16 cast kernels (HBM-bound elementwise work).
//
// Quantisation follows the project spec for the FP8 GEMM inputs: a scale s = amax(|x|) / 448
// per tensor, per 1 x 128 block (A operand: one row, 128 consecutive K) or per 128 x 128 block
// (B operand), and q = e4m3(x / s), rounded to nearest even with saturation at +-448.  The GEMM
// dequantises with q * s.
//
// Layouts: x is row-major [rows, cols] with row stride ldx (elements); q likewise with ldq.
//   per tensor : scales[0]
//   1 x 128    : scales[kb * rows + r]  (block column major, so one k-block's row scales are
//                contiguous for the GEMM epilogue)
//   128 x 128  : scales[rb * ceil(cols / 128) + kb]
#pragma once
#include <cuda_bf16.h>
#include <stdint.h>

namespace cpg {

constexpr float kE4M3Max = 448.0f;
constexpr float kAmaxFloor = 1e-12f;

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

// Two floats -> two E4M3 bytes (lo in the low byte), round to nearest even, saturating.
__device__ __forceinline__ uint16_t cvt_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ uint8_t cvt_e4m3(float v) {
  return static_cast<uint8_t>(cvt_e4m3x2(v, 0.f) & 0xFF);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// x / s for the vector kernels, exact to the E4M3 byte without a division per element.  With
// y = RN(1 / s) (__frcp_rn) and q = RN(x * y), |q - x / s| < ulp(x * y) / 2 + ulp(x / s), so q and
// t = RN(x / s) are at most two fp32 steps apart; e4m3(q) != e4m3(t) (round to nearest even is
// monotone) needs an E4M3 rounding midpoint in between.  Midpoints of the normal E4M3 range
// (>= 2^-6) are the fp32 values whose low 20 fraction bits are 0x80000.  So q whose low bits are
// within 8 steps of that pattern, and nonzero q below 2^-6 (the subnormal E4M3 grid has other
// midpoints), make the whole vector take the IEEE division; all other q give the same byte.
__device__ __forceinline__ bool e4m3_midpoint_risk(float q) {
  const uint32_t b = __float_as_uint(q);
  // Low 20 bits within [0x80000 - 8, 0x80000 + 8] (any exponent: a superset of the normal range),
  // or 0 < |q| < 2^-6 (b << 1 drops the sign: 2 <= 2|q|bits <= 2 * 0x3c7fffff).
  return ((b - 0x7fff8u) & 0xfffffu) <= 16u || (b << 1) - 2u <= 0x78fffffcu;
}

template <int N>
__device__ __forceinline__ void div_by_scale(float (&x)[N], float s, float y) {
  float q[N];
  bool slow = false;
#pragma unroll
  for (int j = 0; j < N; ++j) {
    q[j] = __fmul_rn(x[j], y);
    slow |= e4m3_midpoint_risk(q[j]);
  }
  if (slow) {
#pragma unroll
    for (int j = 0; j < N; ++j) x[j] = x[j] / s;
  } else {
#pragma unroll
    for (int j = 0; j < N; ++j) x[j] = q[j];
  }
}

// N (a multiple of 4) floats already divided by the scale -> N E4M3 bytes, packed 4 per word.
template <int N>
__device__ __forceinline__ void pack_e4m3(const float (&x)[N], uint32_t (&w)[N / 4]) {
#pragma unroll
  for (int i = 0; i < N / 4; ++i) {
    const uint32_t lo = cvt_e4m3x2(x[4 * i], x[4 * i + 1]);
    const uint32_t hi = cvt_e4m3x2(x[4 * i + 2], x[4 * i + 3]);
    w[i] = lo | (hi << 16);
  }
}

// Grid-stride over rows, block-stride over columns (no per-element division).
#define CPG_ROW_LOOP(body)                                                             \
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x)                              \
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) { body; }

// amax over the whole tensor; *amax_bits must be 0 before the launch.  Non-negative floats
// order like their bit patterns, so an integer atomicMax suffices.
template <typename T>
__global__ void amax_kernel(const T* __restrict__ x, int64_t rows, int64_t cols, int64_t ldx,
                            unsigned int* amax_bits) {
  float m = 0.f;
  CPG_ROW_LOOP(m = fmaxf(m, fabsf(to_f32(x[r * ldx + c]))));
  m = warp_max(m);
  __shared__ float red[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (warp == 0) {
    m = lane < static_cast<int>(blockDim.x >> 5) ? red[lane] : 0.f;
    m = warp_max(m);
    if (lane == 0) atomicMax(amax_bits, __float_as_uint(m));
  }
}

// q = e4m3(x / s) with s = max(amax, floor) / 448 read from *amax_bits.
template <typename T>
__global__ void quant_per_tensor_kernel(const T* __restrict__ x, int64_t rows, int64_t cols,
                                        int64_t ldx, uint8_t* __restrict__ q, int64_t ldq,
                                        const unsigned int* amax_bits) {
  const float s = fmaxf(__uint_as_float(*amax_bits), kAmaxFloor) / kE4M3Max;
  CPG_ROW_LOOP(q[r * ldq + c] = cvt_e4m3(to_f32(x[r * ldx + c]) / s));
}

// Vectorised forms of the two per-tensor kernels for rows whose starts and lengths are whole
// 16-byte vectors (8 BF16 or 4 FP32 elements): one 16-byte load per thread and iteration, the
// E4M3 bytes of a vector written at once.  Same per-element arithmetic as the scalar kernels.
template <typename T>
struct Vec16;
template <>
struct Vec16<__nv_bfloat16> {
  static constexpr int kElems = 8;
  __device__ __forceinline__ static void unpack(const uint4& v, float (&f)[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
};
template <>
struct Vec16<float> {
  static constexpr int kElems = 4;
  __device__ __forceinline__ static void unpack(const uint4& v, float (&f)[4]) {
    f[0] = __uint_as_float(v.x);
    f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z);
    f[3] = __uint_as_float(v.w);
  }
};

__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// The first n (< V) elements at p as a 16-byte vector of raw bits, zeros (+0.0) after them.
template <typename T>
__device__ __forceinline__ uint4 ld_partial_vec(const T* p, int n) {
  uint32_t w[4] = {0u, 0u, 0u, 0u};
  if constexpr (sizeof(T) == 2) {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (j < n) w[j >> 1] |= static_cast<uint32_t>(__bfloat16_as_ushort(p[j])) << (16 * (j & 1));
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (j < n) w[j] = __float_as_uint(p[j]);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

template <typename T>
__device__ __forceinline__ float amax_vec(const uint4& raw, float m) {
  float f[Vec16<T>::kElems];
  Vec16<T>::unpack(raw, f);
#pragma unroll
  for (int j = 0; j < Vec16<T>::kElems; ++j) m = fmaxf(m, fabsf(f[j]));
  return m;
}

template <typename T>
__global__ void amax_vec_kernel(const T* __restrict__ x, int64_t rows, int64_t cols, int64_t ldx,
                                unsigned int* amax_bits) {
  constexpr int V = Vec16<T>::kElems;
  const int64_t vcols = cols / V;
  float m = 0.f;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const T* row = x + r * ldx;
#pragma unroll 4
    for (int64_t c = threadIdx.x; c < vcols; c += blockDim.x) {
      float f[V];
      Vec16<T>::unpack(ld_nc_v4(row + c * V), f);
#pragma unroll
      for (int i = 0; i < V; ++i) m = fmaxf(m, fabsf(f[i]));
    }
  }
  m = warp_max(m);
  __shared__ float red[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (warp == 0) {
    m = lane < static_cast<int>(blockDim.x >> 5) ? red[lane] : 0.f;
    m = warp_max(m);
    if (lane == 0) atomicMax(amax_bits, __float_as_uint(m));
  }
}

template <typename T>
__global__ void quant_per_tensor_vec_kernel(const T* __restrict__ x, int64_t rows, int64_t cols,
                                            int64_t ldx, uint8_t* __restrict__ q, int64_t ldq,
                                            const unsigned int* amax_bits) {
  constexpr int V = Vec16<T>::kElems;
  const float s = fmaxf(__uint_as_float(*amax_bits), kAmaxFloor) / kE4M3Max;
  const float y = __frcp_rn(s);
  const int64_t vcols = cols / V;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const T* row = x + r * ldx;
    uint8_t* qrow = q + r * ldq;
#pragma unroll 4
    for (int64_t c = threadIdx.x; c < vcols; c += blockDim.x) {
      float f[V];
      Vec16<T>::unpack(ld_nc_v4(row + c * V), f);
      div_by_scale(f, s, y);
      uint32_t w[V / 4];
      pack_e4m3(f, w);
      if constexpr (V == 8) {
        *reinterpret_cast<uint2*>(qrow + c * V) = make_uint2(w[0], w[1]);
      } else {
        *reinterpret_cast<uint32_t*>(qrow + c * V) = w[0];
      }
    }
  }
}

// Turn the amax bits at *slot into the scale max(amax, floor) / 448, in place.
__global__ void finalize_scale_kernel(unsigned int* slot) {
  const float s = fmaxf(__uint_as_float(*slot), kAmaxFloor) / kE4M3Max;
  *reinterpret_cast<float*>(slot) = s;
}

// 1 x 128 blocks: one warp per (row, 128-column block); lane l owns columns 4l..4l+3.
template <typename T>
__global__ void quant_row_block_kernel(const T* __restrict__ x, int64_t rows, int64_t cols,
                                       int64_t ldx, uint8_t* __restrict__ q, int64_t ldq,
                                       float* __restrict__ scales) {
  const int64_t nkb = (cols + 127) / 128;
  const int64_t warp_id = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp_id >= rows * nkb) return;
  const int64_t r = warp_id / nkb, kb = warp_id - r * nkb;
  float v[4];
  float m = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int64_t c = kb * 128 + 4 * lane + j;
    v[j] = c < cols ? to_f32(x[r * ldx + c]) : 0.f;
    m = fmaxf(m, fabsf(v[j]));
  }
  m = warp_max(m);
  const float s = fmaxf(m, kAmaxFloor) / kE4M3Max;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int64_t c = kb * 128 + 4 * lane + j;
    if (c < cols) q[r * ldq + c] = cvt_e4m3(v[j] / s);
  }
  if (lane == 0) scales[kb * rows + r] = s;
}

// 128 x 128 blocks: one CTA per block (a multiple of 128 threads, at most 512); thread t owns
// column (t & 127) of rows (t >> 7), (t >> 7) + blockDim.x / 128, ...
template <typename T>
__device__ __forceinline__ void quant_tile_block_elems(const T* __restrict__ x, int64_t rows,
                                                       int64_t cols, int64_t ldx,
                                                       uint8_t* __restrict__ q, int64_t ldq,
                                                       float* __restrict__ scales) {
  const int64_t nkb = (cols + 127) / 128;
  const int64_t rb = blockIdx.x / nkb, kb = blockIdx.x - (blockIdx.x / nkb) * nkb;
  const int col = threadIdx.x & 127;
  const int r0 = threadIdx.x >> 7;
  const int rstep = blockDim.x >> 7;
  const int64_t c = kb * 128 + col;
  float m = 0.f;
  for (int rr = r0; rr < 128; rr += rstep) {
    const int64_t r = rb * 128 + rr;
    if (r < rows && c < cols) m = fmaxf(m, fabsf(to_f32(x[r * ldx + c])));
  }
  m = warp_max(m);
  __shared__ float red[16];
  __shared__ float s_sh;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float mm = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) mm = fmaxf(mm, red[w]);
    s_sh = fmaxf(mm, kAmaxFloor) / kE4M3Max;
    scales[rb * nkb + kb] = s_sh;
  }
  __syncthreads();
  const float s = s_sh;
  for (int rr = r0; rr < 128; rr += rstep) {
    const int64_t r = rb * 128 + rr;
    if (r < rows && c < cols) q[r * ldq + c] = cvt_e4m3(to_f32(x[r * ldx + c]) / s);
  }
}

template <typename T>
__global__ void quant_tile_block_kernel(const T* __restrict__ x, int64_t rows, int64_t cols,
                                        int64_t ldx, uint8_t* __restrict__ q, int64_t ldq,
                                        float* __restrict__ scales) {
  quant_tile_block_elems(x, rows, cols, ldx, q, ldq, scales);
}

// 128 x 128 blocks with 16-byte loads: one kTileBlockThreads-thread CTA per block; a thread owns
// one vector (8 BF16 / 4 FP32 columns) of 128 * V / kTileBlockThreads rows and keeps them, packed,
// in registers between the amax and the quantisation, so the block is read once.  Blocks at a
// ragged edge use the element form.
constexpr int kTileBlockThreads = 512;

template <typename T>
__global__ void __launch_bounds__(kTileBlockThreads)
    quant_tile_block_vec_kernel(const T* __restrict__ x, int64_t rows, int64_t cols, int64_t ldx,
                                uint8_t* __restrict__ q, int64_t ldq, float* __restrict__ scales) {
  constexpr int V = Vec16<T>::kElems;
  constexpr int kThreadsPerRow = 128 / V;                             // 16 or 32
  constexpr int kRowsPerPass = kTileBlockThreads / kThreadsPerRow;    // 32 or 16
  constexpr int kPasses = 128 / kRowsPerPass;                         // 4 or 8
  constexpr int kWarps = kTileBlockThreads / 32;
  const int64_t nkb = (cols + 127) / 128;
  const int64_t rb = blockIdx.x / nkb, kb = blockIdx.x - rb * nkb;
  if ((rb + 1) * 128 > rows || (kb + 1) * 128 > cols) {
    quant_tile_block_elems(x, rows, cols, ldx, q, ldq, scales);
    return;
  }
  const int cg = threadIdx.x % kThreadsPerRow;
  const int r0 = threadIdx.x / kThreadsPerRow;
  const T* xp = x + (rb * 128 + r0) * ldx + kb * 128 + cg * V;
  uint8_t* qp = q + (rb * 128 + r0) * ldq + kb * 128 + cg * V;
  uint4 raw[kPasses];
#pragma unroll
  for (int i = 0; i < kPasses; ++i) raw[i] = ld_nc_v4(xp + i * kRowsPerPass * ldx);
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < kPasses; ++i) m = amax_vec<T>(raw[i], m);
  m = warp_max(m);
  __shared__ float red[kWarps];
  __shared__ float s_sh;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float mm = 0.f;
    for (int w = 0; w < kWarps; ++w) mm = fmaxf(mm, red[w]);
    s_sh = fmaxf(mm, kAmaxFloor) / kE4M3Max;
    scales[rb * nkb + kb] = s_sh;
  }
  __syncthreads();
  const float s = s_sh;
  const float y = __frcp_rn(s);
#pragma unroll
  for (int i = 0; i < kPasses; ++i) {
    float v[V];
    Vec16<T>::unpack(raw[i], v);
    div_by_scale(v, s, y);
    uint32_t w[V / 4];
    pack_e4m3(v, w);
    uint8_t* dst = qp + i * kRowsPerPass * ldq;
    if constexpr (V == 8) {
      *reinterpret_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
    } else {
      *reinterpret_cast<uint32_t*>(dst) = w[0];
    }
  }
}

// 1 x 128 blocks with 16-byte loads: lane l holds V consecutive values (8 BF16 / 4 FP32) of a
// block, 128 / V lanes cover one block, and a warp quantises kRowBlockLoads such loads of
// consecutive blocks of one row (8 BF16 / 4 FP32 blocks), issued before the first reduction so
// that each warp keeps kRowBlockLoads 16-byte loads per lane in flight.  Blocks at a ragged right
// edge use element accesses.
constexpr int kRowBlockLoads = 4;

template <typename T>
__host__ __device__ constexpr int row_blocks_per_warp() {
  return kRowBlockLoads * (32 / (128 / Vec16<T>::kElems));
}

template <typename T>
__global__ void quant_row_block_vec_kernel(const T* __restrict__ x, int64_t rows, int64_t cols,
                                           int64_t ldx, uint8_t* __restrict__ q, int64_t ldq,
                                           float* __restrict__ scales) {
  constexpr int V = Vec16<T>::kElems;
  constexpr int kLanesPerBlock = 128 / V;              // 16 or 32
  constexpr int kBlocksPerLoad = 32 / kLanesPerBlock;  // 2 or 1
  constexpr int kPerWarp = row_blocks_per_warp<T>();
  const int64_t nkb = (cols + 127) / 128;
  const int64_t ngroups = (nkb + kPerWarp - 1) / kPerWarp;
  const int64_t warp_id = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp_id >= rows * ngroups) return;  // whole warps
  const int64_t r = warp_id / ngroups;
  const int64_t kb_first = (warp_id - r * ngroups) * kPerWarp + lane / kLanesPerBlock;
  const int li = lane % kLanesPerBlock;
  uint4 raw[kRowBlockLoads];
#pragma unroll
  for (int i = 0; i < kRowBlockLoads; ++i) {
    const int64_t kb = kb_first + i * kBlocksPerLoad;
    const int64_t c0 = kb * 128 + li * V;
    if ((kb + 1) * 128 <= cols) {
      raw[i] = ld_nc_v4(x + r * ldx + c0);
    } else {
      const int64_t n = kb < nkb ? cols - c0 : 0;
      raw[i] = ld_partial_vec(x + r * ldx + c0, n < 0 ? 0 : (n > V ? V : static_cast<int>(n)));
    }
  }
  // Block amax: reductions over each block's lanes, all lanes taking part in every shuffle.
  float m[kRowBlockLoads];
#pragma unroll
  for (int i = 0; i < kRowBlockLoads; ++i) {
    m[i] = amax_vec<T>(raw[i], 0.f);
#pragma unroll
    for (int o = kLanesPerBlock / 2; o > 0; o >>= 1)
      m[i] = fmaxf(m[i], __shfl_xor_sync(0xffffffffu, m[i], o));
  }
#pragma unroll
  for (int i = 0; i < kRowBlockLoads; ++i) {
    const int64_t kb = kb_first + i * kBlocksPerLoad;
    if (kb >= nkb) continue;
    const int64_t c0 = kb * 128 + li * V;
    const float s = fmaxf(m[i], kAmaxFloor) / kE4M3Max;
    float v[V];
    Vec16<T>::unpack(raw[i], v);
    div_by_scale(v, s, __frcp_rn(s));
    if ((kb + 1) * 128 <= cols) {
      uint32_t w[V / 4];
      pack_e4m3(v, w);
      if constexpr (V == 8) {
        *reinterpret_cast<uint2*>(q + r * ldq + c0) = make_uint2(w[0], w[1]);
      } else {
        *reinterpret_cast<uint32_t*>(q + r * ldq + c0) = w[0];
      }
    } else {
#pragma unroll
      for (int j = 0; j < V; ++j)
        if (c0 + j < cols) q[r * ldq + c0 + j] = cvt_e4m3(v[j]);
    }
    if (li == 0) scales[kb * rows + r] = s;
  }
}

// y = bf16(x + bias) for split-K results (x fp32 [rows, cols]).  Vector path when cols, ldx and
// ldy are multiples of 4 and the bases are 16 / 8-byte aligned: each thread converts 4
// consecutive values (one float4 load, one 8-byte store); blockIdx.x walks a row's column
// quads and blockIdx.y (grid-stride) the rows, so there is no per-element division.
__global__ void cast_f32_bf16_kernel(const float* __restrict__ x, int64_t rows, int64_t cols,
                                     int64_t ldx, __nv_bfloat16* __restrict__ y, int64_t ldy,
                                     const __nv_bfloat16* __restrict__ bias) {
  const bool vec = (cols % 4 == 0) && (ldx % 4 == 0) && (ldy % 4 == 0) &&
                   (reinterpret_cast<uintptr_t>(x) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(y) % 8 == 0);
  if (vec) {
    const int64_t c4 = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) * 4;
    if (c4 >= cols) return;
    float b0 = 0.f, b1 = 0.f, b2 = 0.f, b3 = 0.f;
    if (bias != nullptr) {
      b0 = __bfloat162float(bias[c4]);
      b1 = __bfloat162float(bias[c4 + 1]);
      b2 = __bfloat162float(bias[c4 + 2]);
      b3 = __bfloat162float(bias[c4 + 3]);
    }
    for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {
      const float4 v = *reinterpret_cast<const float4*>(x + r * ldx + c4);
      __nv_bfloat162 lo = __floats2bfloat162_rn(v.x + b0, v.y + b1);
      __nv_bfloat162 hi = __floats2bfloat162_rn(v.z + b2, v.w + b3);
      uint2 packed;
      packed.x = *reinterpret_cast<uint32_t*>(&lo);
      packed.y = *reinterpret_cast<uint32_t*>(&hi);
      *reinterpret_cast<uint2*>(y + r * ldy + c4) = packed;
    }
    return;
  }
  // Scalar path: same grid and the same 4 columns per thread, element by element.
  const int64_t c0 = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) * 4;
  for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {
    for (int j = 0; j < 4; ++j) {
      const int64_t c = c0 + j;
      if (c >= cols) break;
      const float b = bias != nullptr ? __bfloat162float(bias[c]) : 0.f;
      y[r * ldy + c] = __float2bfloat16_rn(x[r * ldx + c] + b);
    }
  }
}

#undef CPG_ROW_LOOP

}  // namespace cpg
