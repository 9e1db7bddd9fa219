// Correctly rounded binary32 erf, for the host and the device.
//
// The reference's `gelu_erf` and `erff_map` kernels use a port of the platform
// libm's erff (StablehloMlx/Kernels/Shaders.lean:186-208); this backend instead
// carries the correctly rounded erff, the function the pinned ggml build links
// (CORE-MATH, ref/build.sh:52). It is unique, so it is written here from the
// mathematics:
//
//  * fast path: erf(x) in binary64 by the platform's erf (CUDA's on the device,
//    the C library's on the host -- called, not restated), then rounded to
//    binary32 when no binary32 rounding boundary (a midpoint between adjacent
//    floats) lies within 2^-47 relative of the binary64 value. Both erf
//    implementations are documented to be within a few binary64 ulps
//    (2^-51 relative), far inside that margin.
//  * slow path (about one input in 10^6): erf(x) = 2/sqrt(pi) * sum_n
//    (-1)^n x^(2n+1) / (n! (2n+1)) summed in double-double arithmetic
//    (about 106 bits; at |x| = 4 the alternating terms cancel about 2^17, which
//    leaves about 2^-87 relative error), then rounded the same way.
//  * |x| >= 4: erf(4) > 1 - 2^-25, so the result rounds to +-1.
//  * NaN: the input quieted (what arm64's libm returns, x + x); +-0: itself.
#pragma once
#include <math.h>
#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define SHLO_HD __host__ __device__ __forceinline__
#else
#define SHLO_HD inline
#endif

namespace shlo_erf {

struct dd {
  double hi, lo;
};

SHLO_HD uint32_t f2u(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}
SHLO_HD float u2f(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

// Error-free transformations (Knuth two-sum; two-product with fma).
SHLO_HD dd two_sum(double a, double b) {
  double s = a + b;
  double bb = s - a;
  double e = (a - (s - bb)) + (b - bb);
  return {s, e};
}
SHLO_HD dd quick_two_sum(double a, double b) {
  double s = a + b;
  return {s, b - (s - a)};
}
SHLO_HD dd two_prod(double a, double b) {
  double p = a * b;
  return {p, fma(a, b, -p)};
}
SHLO_HD dd dd_add(dd a, dd b) {
  dd s = two_sum(a.hi, b.hi);
  dd t = two_sum(a.lo, b.lo);
  s.lo += t.hi;
  s = quick_two_sum(s.hi, s.lo);
  s.lo += t.lo;
  return quick_two_sum(s.hi, s.lo);
}
SHLO_HD dd dd_mul(dd a, dd b) {
  dd p = two_prod(a.hi, b.hi);
  p.lo += a.hi * b.lo + a.lo * b.hi;
  return quick_two_sum(p.hi, p.lo);
}
SHLO_HD dd dd_div_d(dd a, double b) {
  double q1 = a.hi / b;
  dd p = two_prod(q1, b);
  double s = (a.hi - p.hi) - p.lo + a.lo;
  double q2 = s / b;
  return quick_two_sum(q1, q2);
}

// Round `y` (an approximation with relative error below 2^-tol_log2) to binary32;
// returns false when a rounding boundary lies within the error bound.
SHLO_HD bool round_certain(double y, int tol_log2, float *out) {
  float f = (float)y;  // round to nearest even, with subnormals
  float lo = nextafterf(f, -INFINITY), hi = nextafterf(f, INFINITY);
  double mlo = 0.5 * ((double)f + (double)lo), mhi = 0.5 * ((double)f + (double)hi);
  double tol = fabs(y) * ldexp(1.0, -tol_log2);
  if (fabs(y - mlo) <= tol || fabs(y - mhi) <= tol) return false;
  *out = f;
  return true;
}

// 2/sqrt(pi) as a double-double (from a binary128 evaluation).
#define SHLO_TWO_OVER_SQRTPI_HI 0x1.20dd750429b6dp+0
#define SHLO_TWO_OVER_SQRTPI_LO 0x1.1ae3a914fed8p-56

// erf(a) for 0 < a < 4 in double-double, by its Maclaurin series.
SHLO_HD dd erf_series(double a) {
  dd x2 = two_prod(a, a);
  dd term = {a, 0.0};  // a^(2n+1) / n!
  dd sum = term;
  for (int n = 1; n < 160; n++) {
    term = dd_div_d(dd_mul(term, x2), (double)n);
    dd c = dd_div_d(term, (double)(2 * n + 1));
    if (n & 1) c = {-c.hi, -c.lo};
    sum = dd_add(sum, c);
    if (fabs(c.hi) < ldexp(a, -112)) break;
  }
  return dd_mul(sum, dd{SHLO_TWO_OVER_SQRTPI_HI, SHLO_TWO_OVER_SQRTPI_LO});
}

// The slow path alone (used by the exhaustive self-check as an independent method).
SHLO_HD float erff_slow(float x) {
  uint32_t b = f2u(x);
  uint32_t m = b & 0x7FFFFFFFu;
  if (m > 0x7F800000u) return u2f(b | 0x00400000u);
  if (m == 0) return x;
  float a = u2f(m);
  float r;
  if (a >= 4.0f) {
    r = 1.0f;
  } else {
    dd s = erf_series((double)a);
    double y = s.hi + s.lo;
    if (!round_certain(y, 80, &r)) r = (float)y;  // never observed: |y - midpoint| > 2^-80 |y|
  }
  return (b >> 31) ? -r : r;
}

// Correctly rounded erff. `erf64` is the platform's binary64 erf.
SHLO_HD float erff_cr(float x) {
  uint32_t b = f2u(x);
  uint32_t m = b & 0x7FFFFFFFu;
  if (m > 0x7F800000u) return u2f(b | 0x00400000u);
  if (m == 0) return x;
  float a = u2f(m);
  if (a >= 4.0f) return (b >> 31) ? -1.0f : 1.0f;
  float r;
  if (!round_certain(erf((double)a), 47, &r)) r = erff_slow(a);
  return (b >> 31) ? -r : r;
}

}  // namespace shlo_erf
