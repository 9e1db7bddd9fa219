// Scalar helpers shared by the exact kernels: bit casts, arm64's default NaN,
// and ggml-cpu's NEON exp.
#pragma once
#include <cstdint>

#include "common.cuh"

namespace shlo {

__device__ __forceinline__ uint32_t fbits(float f) { return __float_as_uint(f); }
__device__ __forceinline__ float bitsf(uint32_t u) { return __uint_as_float(u); }

// arm64's default NaN, what an invalid operation (inf*0, inf-inf, 0/0) gives
// there (FPCR.DN clear produces it for invalid operations; the GPU's own NaN is
// 0x7FFFFFFF). The reductions return it for every NaN result.
__device__ __forceinline__ float arm_nan(float v) { return v != v ? __uint_as_float(0x7FC00000u) : v; }

// ggml_v_expf, one lane (StablehloMlx/Kernels/Math.lean:28-49): ggml-cpu's NEON
// exp ("adapted from arm limited optimized routine"), with vfmaq_f32(a, b, c)
// = fma(b, c, a) and vfmsq_f32(a, b, c) = fma(-b, c, a).
__device__ __forceinline__ float ggml_v_expf(float x) {
  const float r = bitsf(0x4B400000u);
  float z = __fmaf_rn(x, bitsf(0x3FB8AA3Bu), r);
  float n = __fsub_rn(z, r);
  float b = __fmaf_rn(-n, bitsf(0x35BFBE8Eu), __fmaf_rn(-n, bitsf(0x3F317200u), x));
  uint32_t e = fbits(z) << 23;
  float k = bitsf(e + 0x3F800000u);
  float u = __fmul_rn(b, b);
  float p1 = __fmaf_rn(bitsf(0x3E2AAF33u), b, bitsf(0x3EFFFEDBu));
  float p2 = __fmaf_rn(bitsf(0x3C072010u), b, bitsf(0x3D2B9F17u));
  float p3 = __fmaf_rn(p2, u, p1);
  float j = __fmaf_rn(p3, u, __fmul_rn(bitsf(0x3F7FFFF6u), b));
  float an = fabsf(n);
  uint32_t d = (n <= 0.0f) ? 0x82000000u : 0u;
  float s1 = bitsf(d + 0x7F000000u);
  if (an > bitsf(0x43400000u)) return __fmul_rn(s1, s1);
  if (an > bitsf(0x42FC0000u)) {
    float s2 = bitsf(e - d);
    return __fmul_rn(__fmaf_rn(s2, j, s2), s1);
  }
  return __fmaf_rn(k, j, k);
}

}  // namespace shlo
