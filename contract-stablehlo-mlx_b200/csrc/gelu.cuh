// gelu_erf's arithmetic (StablehloMlx/Kernels/Shaders.lean:186-199,
// ggml_vec_gelu_erf_f32): y = (0.5f*x) * (1.0f + erff(x*SQRT_2_INV)) with the
// correctly rounded erff; a NaN input returns itself quieted, as every arm64
// step does. Shared by the standalone kernel (ggml_kernels.cu) and mul_mat's
// fused epilogue (mul_mat.cuh).
#pragma once
#include "erff_cr.cuh"
#include "ggml_math.cuh"

namespace shlo {

__device__ __forceinline__ float gelu_nan(float v, float r) {
  const uint32_t b = fbits(v);
  if ((b & 0x7FFFFFFFu) > 0x7F800000u) return bitsf(b | 0x00400000u);
  if (r != r) return bitsf(0x7FC00000u);  // -inf * 0: arm64's default NaN
  return r;
}

__device__ __forceinline__ float gelu_of(float v, float ev) {
  return __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, ev));
}

// Four values: erff's Taylor path as straight-line code for the four, then the
// NaN rules for the values erff took out of that path (an infinite or NaN input
// is out of its range; for the rest the product is finite). The binary32 steps
// run two values a packed instruction, each lane the scalar operation.
__device__ __forceinline__ float4 gelu4(float4 v4, const shlo_erf::ErfSmem *t) {
  const float2 v01 = make_float2(v4.x, v4.y), v23 = make_float2(v4.z, v4.w);
  const float2 k = make_float2(bitsf(0x3F3504F3u), bitsf(0x3F3504F3u));
  const float2 x01 = __fmul2_rn(v01, k), x23 = __fmul2_rn(v23, k);
  const float x[4] = {x01.x, x01.y, x23.x, x23.y};
  float ev[4];
  const unsigned rare = shlo_erf::erff4_smem(x, ev, t);
  const float2 h = make_float2(0.5f, 0.5f), one = make_float2(1.0f, 1.0f);
  const float2 r01 = __fmul2_rn(__fmul2_rn(h, v01), __fadd2_rn(one, make_float2(ev[0], ev[1])));
  const float2 r23 = __fmul2_rn(__fmul2_rn(h, v23), __fadd2_rn(one, make_float2(ev[2], ev[3])));
  float r[4] = {r01.x, r01.y, r23.x, r23.y};
  if (rare) {
    const float v[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
    for (int i = 0; i < 4; i++)
      if (rare & (1u << i)) r[i] = gelu_nan(v[i], r[i]);
  }
  return make_float4(r[0], r[1], r[2], r[3]);
}

}  // namespace shlo
