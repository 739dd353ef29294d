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
  const int64_t vcols = cols / V;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const T* row = x + r * ldx;
    uint8_t* qrow = q + r * ldq;
#pragma unroll 4
    for (int64_t c = threadIdx.x; c < vcols; c += blockDim.x) {
      float f[V];
      Vec16<T>::unpack(ld_nc_v4(row + c * V), f);
      uint32_t w[V / 4];
#pragma unroll
      for (int i = 0; i < V / 4; ++i) {
        const uint32_t lo = cvt_e4m3x2(f[4 * i] / s, f[4 * i + 1] / s);
        const uint32_t hi = cvt_e4m3x2(f[4 * i + 2] / s, f[4 * i + 3] / s);
        w[i] = lo | (hi << 16);
      }
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

// 128 x 128 blocks: one 256-thread CTA per block; thread t owns column (t & 127) of rows
// (t >> 7), (t >> 7) + 2, ... (64 values).
template <typename T>
__global__ void quant_tile_block_kernel(const T* __restrict__ x, int64_t rows, int64_t cols,
                                        int64_t ldx, uint8_t* __restrict__ q, int64_t ldq,
                                        float* __restrict__ scales) {
  const int64_t nkb = (cols + 127) / 128;
  const int64_t rb = blockIdx.x / nkb, kb = blockIdx.x - (blockIdx.x / nkb) * nkb;
  const int col = threadIdx.x & 127;
  const int r0 = threadIdx.x >> 7;
  const int64_t c = kb * 128 + col;
  float m = 0.f;
  for (int rr = r0; rr < 128; rr += 2) {
    const int64_t r = rb * 128 + rr;
    if (r < rows && c < cols) m = fmaxf(m, fabsf(to_f32(x[r * ldx + c])));
  }
  m = warp_max(m);
  __shared__ float red[8];
  __shared__ float s_sh;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float mm = 0.f;
    for (int w = 0; w < 8; ++w) mm = fmaxf(mm, red[w]);
    s_sh = fmaxf(mm, kAmaxFloor) / kE4M3Max;
    scales[rb * nkb + kb] = s_sh;
  }
  __syncthreads();
  const float s = s_sh;
  for (int rr = r0; rr < 128; rr += 2) {
    const int64_t r = rb * 128 + rr;
    if (r < rows && c < cols) q[r * ldq + c] = cvt_e4m3(to_f32(x[r * ldx + c]) / s);
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
