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

// sin(x) and cos(x) for |x| <= kSinCosFastRange in float, within 0.75 ulp(1) of absolute error
// (checked on the host against double sin/cos over 8 million points of [-8192, 8192]).
//
// Method (Cody and Waite, "Software Manual for the Elementary Functions", 1980): reduce by pi/2,
// x = k pi/2 + r with |r| <= pi/4, where pi/2 = HI + MID + LO and HI, MID carry 12 significant bits
// each, so k*HI and k*MID are exact for |k| < 4096 and x - k*HI is exact (Sterbenz).  k is the
// round-to-nearest of x*2/pi read from the low mantissa bits of x*2/pi + 1.5*2^23, whose last two
// bits are k mod 4 (the quadrant).  sin(r) and cos(r) are the Taylor series through r^9 and r^10
// (coefficients (-1)^n/n!); on |r| <= pi/4 their truncation errors are below
// (pi/4)^11/11! = 1.8e-9 and (pi/4)^12/12! = 1.2e-10, and neither sum cancels.  The quadrant then
// swaps and negates: (s, c) = (sr, cr), (cr, -sr), (-sr, -cr), (-cr, sr) for k mod 4 = 0..3.
// The constants were computed from pi to 60 digits (the split) and from 1/n! (the series).
CUFKB_HD void sincos_fast(float x, float& s, float& c) {
  constexpr float kTwoOverPi = 0.6366197466850281f;
  constexpr float kShifter = 12582912.0f;  // 1.5 * 2^23
  constexpr float kHi = 1.57080078125f;
  constexpr float kMid = -4.453584551811218e-06f;
  constexpr float kLo = -8.705515752716053e-10f;
  const float t = fmaf(x, kTwoOverPi, kShifter);
  const float k = t - kShifter;
  float r = fmaf(-k, kHi, x);
  r = fmaf(-k, kMid, r);
  r = fmaf(-k, kLo, r);
  const float r2 = r * r;
  float p = 2.7557318844628753e-06f;
  p = fmaf(p, r2, -0.00019841270113829523f);
  p = fmaf(p, r2, 0.008333333767950535f);
  p = fmaf(p, r2, -0.1666666716337204f);
  const float sr = fmaf(p, r * r2, r);
  float q = -2.755731998149713e-07f;
  q = fmaf(q, r2, 2.4801587642286904e-05f);
  q = fmaf(q, r2, -0.0013888889225199819f);
  q = fmaf(q, r2, 0.0416666679084301f);
  q = fmaf(q, r2, -0.5f);
  const float cr = fmaf(q, r2, 1.0f);
  const uint32_t quadrant = f2u(t);
  const bool swap = (quadrant & 1u) != 0u;
  const float ss = swap ? cr : sr;
  const float cc = swap ? sr : cr;
  s = u2f(f2u(ss) ^ ((quadrant & 2u) << 30));
  c = u2f(f2u(cc) ^ (((quadrant + 1u) & 2u) << 30));
}

#if defined(__CUDACC__)
// The same computation on two independent arguments with Blackwell's packed FP32 instructions
// (fma/mul/add .f32x2): every multiply-add above becomes one instruction for both lanes, and each
// lane's result is bit-identical to sincos_fast on that lane.  Device code for sm_100 and later.
__device__ __forceinline__ void sincos_fast2(float2 x, float2& s, float2& c) {
  const float2 two_over_pi = make_float2(0.6366197466850281f, 0.6366197466850281f);
  const float2 shifter = make_float2(12582912.0f, 12582912.0f);
  const float2 neg_shifter = make_float2(-12582912.0f, -12582912.0f);
  const float2 neg_hi = make_float2(-1.57080078125f, -1.57080078125f);
  const float2 neg_mid = make_float2(4.453584551811218e-06f, 4.453584551811218e-06f);
  const float2 neg_lo = make_float2(8.705515752716053e-10f, 8.705515752716053e-10f);
  const float2 t = __ffma2_rn(x, two_over_pi, shifter);
  const float2 k = __fadd2_rn(t, neg_shifter);
  float2 r = __ffma2_rn(k, neg_hi, x);
  r = __ffma2_rn(k, neg_mid, r);
  r = __ffma2_rn(k, neg_lo, r);
  const float2 r2 = __fmul2_rn(r, r);
  float2 p = make_float2(2.7557318844628753e-06f, 2.7557318844628753e-06f);
  p = __ffma2_rn(p, r2, make_float2(-0.00019841270113829523f, -0.00019841270113829523f));
  p = __ffma2_rn(p, r2, make_float2(0.008333333767950535f, 0.008333333767950535f));
  p = __ffma2_rn(p, r2, make_float2(-0.1666666716337204f, -0.1666666716337204f));
  const float2 sr = __ffma2_rn(p, __fmul2_rn(r, r2), r);
  float2 q = make_float2(-2.755731998149713e-07f, -2.755731998149713e-07f);
  q = __ffma2_rn(q, r2, make_float2(2.4801587642286904e-05f, 2.4801587642286904e-05f));
  q = __ffma2_rn(q, r2, make_float2(-0.0013888889225199819f, -0.0013888889225199819f));
  q = __ffma2_rn(q, r2, make_float2(0.0416666679084301f, 0.0416666679084301f));
  q = __ffma2_rn(q, r2, make_float2(-0.5f, -0.5f));
  const float2 cr = __ffma2_rn(q, r2, make_float2(1.0f, 1.0f));
  const uint32_t qx = f2u(t.x), qy = f2u(t.y);
  const float sx = (qx & 1u) ? cr.x : sr.x, cx = (qx & 1u) ? sr.x : cr.x;
  const float sy = (qy & 1u) ? cr.y : sr.y, cy = (qy & 1u) ? sr.y : cr.y;
  s = make_float2(u2f(f2u(sx) ^ ((qx & 2u) << 30)), u2f(f2u(sy) ^ ((qy & 2u) << 30)));
  c = make_float2(u2f(f2u(cx) ^ (((qx + 1u) & 2u) << 30)), u2f(f2u(cy) ^ (((qy + 1u) & 2u) << 30)));
}
#endif

}  // namespace cufkb
