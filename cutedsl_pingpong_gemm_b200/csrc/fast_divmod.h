// FastDivmod: division by a runtime-invariant divisor with one multiply-high and one shift.
//
// Same arithmetic as the reference's FastDivmod (fast_math.py:49-81): for a divisor d,
//   p          = 31 + ceil(log2(d))                         (fast_math.py:61, find_log2 :29-31)
//   multiplier = ceil(2^p / d) mod 2^32                     (fast_math.py:63)
//   shift      = p - 32 (mod 2^32)                          (fast_math.py:64)
//   div(x)     = umulhi(x, multiplier) >> shift, or x when d == 1   (fast_math.py:72-76)
//   divmod(x)  = (q, x - q * d)                             (fast_math.py:78-81)
// This is the round-up multiply-shift method of Granlund & Montgomery ("Division by invariant
// integers using multiplication", PLDI 1994); it is exact for 0 <= x < 2^31 and 1 <= d < 2^31.
//
// The same header is compiled into the host library (scheduler parameters, tile maps) and into
// the device kernels (tile coordinates), so host and device share one implementation.
#pragma once
#include <stdint.h>

#if defined(__CUDACC__)
#define CPG_HD __host__ __device__ __forceinline__
#else
#define CPG_HD inline
#endif

namespace cpg {

struct FastDivmod {
  int32_t divisor;
  uint32_t multiplier;
  uint32_t shift_right;
};

// Leading-zero count of a 32-bit value (32 for zero), portable between host and device.
CPG_HD int32_t clz32(uint32_t x) {
#if defined(__CUDA_ARCH__)
  return __clz(x);
#else
  return x == 0 ? 32 : __builtin_clz(x);
#endif
}

// ceil(log2(x)) for x >= 1 (fast_math.py:29-31).
CPG_HD int32_t find_log2(int32_t x) {
  int32_t a = 31 - clz32(static_cast<uint32_t>(x));
  return a + ((x & (x - 1)) != 0 ? 1 : 0);
}

CPG_HD uint32_t umulhi32(uint32_t a, uint32_t b) {
#if defined(__CUDA_ARCH__)
  return __umulhi(a, b);
#else
  return static_cast<uint32_t>((static_cast<uint64_t>(a) * static_cast<uint64_t>(b)) >> 32);
#endif
}

// Host-side parameter computation (also usable on device).  divisor must be >= 1.
CPG_HD FastDivmod fast_divmod_create(int32_t divisor) {
  FastDivmod f;
  uint32_t p = static_cast<uint32_t>(31 + find_log2(divisor));
  uint64_t d = static_cast<uint32_t>(divisor);
  f.divisor = divisor;
  f.multiplier = static_cast<uint32_t>(((uint64_t(1) << p) + d - 1) / d);
  f.shift_right = p - 32u;  // wraps for divisor 1; div() bypasses it then
  return f;
}

CPG_HD int32_t fast_div(const FastDivmod& f, int32_t x) {
  if (f.divisor == 1) return x;
  return static_cast<int32_t>(umulhi32(static_cast<uint32_t>(x), f.multiplier) >> f.shift_right);
}

CPG_HD void fast_divmod(const FastDivmod& f, int32_t x, int32_t& q, int32_t& r) {
  q = fast_div(f, x);
  r = x - q * f.divisor;
}

}  // namespace cpg
