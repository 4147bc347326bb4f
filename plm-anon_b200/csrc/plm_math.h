// Elementary functions with a fixed, fully specified sequence of IEEE single-precision operations.
//
// The verify decode (Voronoi assignment) and the relaxed acceptance rules must give bit-identical results on the
// GPU and in the CPU oracle for identical fp32 logits. Library expf/logf differ between the two sides in the last
// bit, so this file defines its own:
//
//   plm_expf  Cody & Waite argument reduction x = n ln2 + r (ln2 split into a 15-bit head and a tail, so n * head
//             is exact), e^r by its Taylor series to degree 7 (coefficients 1/k!, truncation error < 0.1 ulp for
//             |r| <= ln2 / 2), then scaling by 2^n built from the exponent bits.
//   plm_logf  x = m 2^e with m in [sqrt(1/2), sqrt(2)), log m = 2 atanh(s) with s = (m - 1) / (m + 1), by the odd
//             series 2 s (1 + s^2/3 + s^4/5 + ... + s^10/11) (truncation < 1e-10 relative), plus e ln2.
//
// Every step is a separate add, multiply, divide, rint or bit operation: the translation unit that uses these on
// the GPU is compiled with -fmad=false, and numpy float32 arithmetic performs the same steps, so both sides round
// identically. The coefficients are written as hexadecimal literals (the float32 values of 1/k!, 1/(2j+1)).
// Accuracy against float64 is checked by the CPU test suite (<= 2 ulp over the ranges the round uses).
#pragma once

#include <math.h>
#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define PLM_HD __host__ __device__ __forceinline__
#else
#define PLM_HD static inline
#endif

namespace plm_math {

PLM_HD float bits_to_float(uint32_t b) {
#if defined(__CUDA_ARCH__)
  return __uint_as_float(b);
#else
  float f;
  memcpy(&f, &b, 4);
  return f;
#endif
}

PLM_HD uint32_t float_to_bits(float f) {
#if defined(__CUDA_ARCH__)
  return __float_as_uint(f);
#else
  uint32_t b;
  memcpy(&b, &f, 4);
  return b;
#endif
}

constexpr float kLn2Hi = 0x1.62e4p-1f;        // 22713 / 32768, 15 significant bits
constexpr float kLn2Lo = 0x1.7f7d1cp-20f;     // ln 2 - kLn2Hi
constexpr float kLog2e = 0x1.715476p+0f;      // 1 / ln 2
constexpr float kExpMaxArg = 0x1.62e43p+6f;   // 88.72283935546875: above this e^x overflows
constexpr float kExpMinArg = -0x1.9fe36ap+6f; // -103.972084...: below this e^x rounds to zero

PLM_HD float plm_expf(float x) {
  if (!(x == x)) return x;
  if (x > kExpMaxArg) return INFINITY;
  if (x < kExpMinArg) return 0.0f;
  const float n = rintf(x * kLog2e);
  const float r = (x - n * kLn2Hi) - n * kLn2Lo;
  float p = 0x1.a01a02p-13f;  // 1/7!
  p = p * r + 0x1.6c16c2p-10f;  // 1/6!
  p = p * r + 0x1.111112p-7f;   // 1/5!
  p = p * r + 0x1.555556p-5f;   // 1/4!
  p = p * r + 0x1.555556p-3f;   // 1/3!
  p = p * r + 0x1.0p-1f;        // 1/2!
  p = p * r + 1.0f;
  p = p * r + 1.0f;
  int ni = int(n);
  if (ni > 127) {
    p = p * 0x1.0p127f;
    ni -= 127;
  }
  if (ni < -126) {
    p = p * 0x1.0p-126f;
    ni += 126;
  }
  return p * bits_to_float(uint32_t(ni + 127) << 23);
}

PLM_HD float plm_logf(float x) {
  if (!(x == x) || x < 0.0f) return NAN;
  if (x == 0.0f) return -INFINITY;
  if (x == INFINITY) return x;
  int e = 0;
  uint32_t b = float_to_bits(x);
  if (b < 0x00800000u) {  // subnormal: scale into the normal range first
    x = x * 0x1.0p23f;
    b = float_to_bits(x);
    e = -23;
  }
  e += int(b >> 23) - 127;
  float m = bits_to_float((b & 0x007FFFFFu) | 0x3F800000u);  // [1, 2)
  if (m > 0x1.6a09e6p+0f) {                                  // sqrt(2)
    m = m * 0.5f;
    e += 1;
  }
  const float s = (m - 1.0f) / (m + 1.0f);
  const float z = s * s;
  float p = 0x1.745d18p-4f;  // 1/11
  p = p * z + 0x1.c71c72p-4f;  // 1/9
  p = p * z + 0x1.24924ap-3f;  // 1/7
  p = p * z + 0x1.99999ap-3f;  // 1/5
  p = p * z + 0x1.555556p-2f;  // 1/3
  p = p * z + 1.0f;
  const float lm = (2.0f * s) * p;
  const float fe = float(e);
  return fe * kLn2Hi + (fe * kLn2Lo + lm);
}

// Monotone unsigned key of a float: larger floats give larger keys (used for the top-m radix select).
PLM_HD uint32_t orderable_key(float x) {
  const uint32_t b = float_to_bits(x);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// The condensed-problem key of the Voronoi engine: the cost's bits mapped to an order-preserving signed integer,
// low 7 bits replaced by the target index (plm/iterate.py:101-102).
PLM_HD int32_t condense_key(float cost, int target) {
  const int32_t b = int32_t(float_to_bits(cost));
  const int32_t ordered = b >= 0 ? b : (b ^ 0x7FFFFFFF);
  return (ordered & ~0x7F) | target;
}

// Inverse of condense_key's cost part (plm/iterate.py:132-134): the cost with its low 7 mantissa bits cleared.
PLM_HD float condensed_cost(int32_t key) {
  const int32_t carried = key & ~0x7F;
  return bits_to_float(uint32_t(carried >= 0 ? carried : (carried ^ 0x7FFFFFFF)));
}

}  // namespace plm_math
