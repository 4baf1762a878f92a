// Scalar math shared by the kernels; compiles for the device (nvcc) and for the host (g++, used by
// the CPU accuracy test of the sine/cosine below).
#pragma once

#include <cmath>
#include <cstdint>
#include <cstring>

#if defined(__CUDACC__)
#define CUFKB_HD __host__ __device__ __forceinline__
#else
#define CUFKB_HD inline
#endif

namespace cufkb {

CUFKB_HD uint32_t f2u(float x) {
#if defined(__CUDA_ARCH__)
  return __float_as_uint(x);
#else
  uint32_t u;
  std::memcpy(&u, &x, sizeof u);
  return u;
#endif
}

CUFKB_HD float u2f(uint32_t u) {
#if defined(__CUDA_ARCH__)
  return __uint_as_float(u);
#else
  float x;
  std::memcpy(&x, &u, sizeof x);
  return x;
#endif
}

// Largest |x| served by the reduction below; beyond it the caller falls back to the library call.
constexpr float kSinCosFastRange = 8192.0f;

// sin(x) and cos(x) for |x| <= kSinCosFastRange in float, within 1.1 ulp(1) of absolute error
// (checked on the host against double sin/cos over millions of points of [-8192, 8192]).
//
// Method: Cody and Waite's additive reduction ("Software Manual for the Elementary Functions",
// 1980), here by pi rather than pi/2: x = k pi + r with |r| <= pi/2, where pi = HI + LO, HI carries
// 12 significant bits, so k*HI is exact for |k| < 4096 and x - k*HI is exact (Sterbenz), and LO is
// pi - HI rounded to float (off by 3.3e-13, i.e. at most 1e-9 at |k| = 4096), so the reduction
// rounds once.  k is the round-to-nearest of x/pi, read from the low mantissa bits of
// x/pi + 1.5*2^23, whose last bit is k mod 2.  Then sin x = (-1)^k sin r and cos x = (-1)^k cos r:
// one sign flip, no quadrant swap.  sin r = r + r^3 P(r^2) (P of degree 3) and cos r = 1 + r^2 Q(r^2)
// (Q of degree 4) are minimax polynomials for the absolute error on |r| <= pi/2, computed for this
// file with the Remez exchange algorithm in 50-digit arithmetic (errors 4.6e-9 and 2.4e-10 before
// rounding the coefficients to float).  Neither sum cancels except cos r near |r| = pi/2, where the
// absolute error stays near 1 ulp(1).  The pi split was taken from pi to 50 digits.
CUFKB_HD void sincos_fast(float x, float& s, float& c) {
  constexpr float kOneOverPi = 0.31830987334251404f;
  constexpr float kShifter = 12582912.0f;  // 1.5 * 2^23
  constexpr float kHi = 3.1416015625f;
  constexpr float kLo = -8.90890987648163e-06f;
  const float t = fmaf(x, kOneOverPi, kShifter);
  const float k = t - kShifter;
  float r = fmaf(-k, kHi, x);
  r = fmaf(-k, kLo, r);
  const float r2 = r * r;
  float p = 2.6000548132287804e-06f;
  p = fmaf(p, r2, -0.00019806614727713168f);
  p = fmaf(p, r2, 0.008333017118275166f);
  p = fmaf(p, r2, -0.16666656732559204f);
  const float sr = fmaf(p * r2, r, r);
  float q = -2.607710598567792e-07f;
  q = fmaf(q, r2, 2.4761886379565112e-05f);
  q = fmaf(q, r2, -0.00138884037733078f);
  q = fmaf(q, r2, 0.04166664183139801f);
  q = fmaf(q, r2, -0.5f);
  const float cr = fmaf(q, r2, 1.0f);
  const uint32_t sign = f2u(t) << 31;  // (k mod 2) in the sign bit
  s = u2f(f2u(sr) ^ sign);
  c = u2f(f2u(cr) ^ sign);
}

#if defined(__CUDACC__)
// The same computation on two independent arguments with Blackwell's packed FP32 instructions
// (fma/mul/add .f32x2): every multiply-add above becomes one instruction for both lanes, and each
// lane's result is bit-identical to sincos_fast on that lane.  Device code for sm_100 and later.
__device__ __forceinline__ void sincos_fast2(float2 x, float2& s, float2& c) {
  const float2 one_over_pi = make_float2(0.31830987334251404f, 0.31830987334251404f);
  const float2 shifter = make_float2(12582912.0f, 12582912.0f);
  const float2 neg_shifter = make_float2(-12582912.0f, -12582912.0f);
  const float2 neg_hi = make_float2(-3.1416015625f, -3.1416015625f);
  const float2 neg_lo = make_float2(8.90890987648163e-06f, 8.90890987648163e-06f);
  const float2 t = __ffma2_rn(x, one_over_pi, shifter);
  const float2 k = __fadd2_rn(t, neg_shifter);
  float2 r = __ffma2_rn(k, neg_hi, x);
  r = __ffma2_rn(k, neg_lo, r);
  const float2 r2 = __fmul2_rn(r, r);
  float2 p = make_float2(2.6000548132287804e-06f, 2.6000548132287804e-06f);
  p = __ffma2_rn(p, r2, make_float2(-0.00019806614727713168f, -0.00019806614727713168f));
  p = __ffma2_rn(p, r2, make_float2(0.008333017118275166f, 0.008333017118275166f));
  p = __ffma2_rn(p, r2, make_float2(-0.16666656732559204f, -0.16666656732559204f));
  const float2 sr = __ffma2_rn(__fmul2_rn(p, r2), r, r);
  float2 q = make_float2(-2.607710598567792e-07f, -2.607710598567792e-07f);
  q = __ffma2_rn(q, r2, make_float2(2.4761886379565112e-05f, 2.4761886379565112e-05f));
  q = __ffma2_rn(q, r2, make_float2(-0.00138884037733078f, -0.00138884037733078f));
  q = __ffma2_rn(q, r2, make_float2(0.04166664183139801f, 0.04166664183139801f));
  q = __ffma2_rn(q, r2, make_float2(-0.5f, -0.5f));
  const float2 cr = __ffma2_rn(q, r2, make_float2(1.0f, 1.0f));
  const uint32_t sx = f2u(t.x) << 31, sy = f2u(t.y) << 31;
  s = make_float2(u2f(f2u(sr.x) ^ sx), u2f(f2u(sr.y) ^ sy));
  c = make_float2(u2f(f2u(cr.x) ^ sx), u2f(f2u(cr.y) ^ sy));
}
#endif

}  // namespace cufkb
