// mul_mat for small products (few rows, few tiles: a batch of one, the
// timestep MLP), ggml_vec_dot_f32 bit for bit.
//
// The packed-segment layout of mul_mat.cuh puts leaf s of ggml's reduction
// tree (one class of the sixteen k-ascending chains) in the s-th contiguous
// segment of the packed K axis. The sixteen chains of an output are
// independent until the tree adds them, so here they run side by side: a CTA
// owns a 32 m x 32 r tile over the whole K, and warp w computes the chains of
// segments 2w and 2w + 1 for every output of the tile (one lane: 8 m x 4 r,
// paired FP32 FMAs), adding them as the tree's lowest pair (the older segment
// on the left). The eight pair sums of each output then meet in shared memory
// and one thread adds the rest of the tree, ((P0+P1)+(P2+P3))+((P4+P5)+(P6+P7)),
// then the tail (K mod 16, in ggml's order), the NaN rule and the fused adds.
// Nothing is parked in global memory, and a grid of 32 x 32 tiles fills the GPU
// where 128 x 128 tiles would leave most SMs idle.
//
// Each warp streams its own segments through a private ring of NS stages of
// 4 packed k rows (cp.async: a stage is 4 rows x 16 copies of 16 bytes, two a
// lane), synchronising only within the warp.
#define SHLO_MUL_MAT_INSTANCES
#include "mul_mat.cuh"

namespace shlo {
namespace sg {
constexpr int NS = 4;                   // stages a warp
constexpr int ROW = TM + TR;            // floats of one packed k row of the tile (w then x)
constexpr int STAGE = 4 * ROW;          // 4 k rows
constexpr int WARP_FLOATS = NS * STAGE;
constexpr int SMEM_FLOATS = 8 * WARP_FLOATS;  // the rings; then the pair sums (8 warps x 512 float2)
static_assert(SMEM_FLOATS >= 8 * 512 * 2, "the pair sums fit where the rings were");
}  // namespace sg

template <bool EPI>
__global__ void __launch_bounds__(sg::THREADS, 2) k_mul_mat_seg(MMArgs a) {
  using namespace sg;
  __shared__ __align__(16) float smem[SMEM_FLOATS];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mtiles = a.Mp / TM;
  const int m0 = (blockIdx.x % mtiles) * TM;
  const int rb = blockIdx.x / mtiles;
  const int bx = rb / a.r_tiles;
  const int64_t rl0 = (int64_t)(rb % a.r_tiles) * TR;
  const int64_t Kq = 16 * (int64_t)a.segp;
  const float *wp = a.wp + (a.wbs ? (int64_t)bx * Kq * a.Mp : 0) + m0;
  const float *xp = a.xp + (int64_t)bx * Kq * a.Np + rl0;
  float *ring = smem + warp * WARP_FLOATS;
  const int mo = (lane & 3) * 8, ro = (lane >> 2) * 4;
  const int groups = a.segp / 4;  // stages of a segment

  float2 pair[16];
#pragma unroll 1
  for (int h = 0; h < 2; h++) {
    const int64_t k0 = (int64_t)(2 * warp + h) * a.segp;  // the segment's first packed k row
    // copy c = lane + 32 t of stage g: k row c / 16, 16 bytes c % 16 of the
    // row (w for 0..7, x for 8..15)
    auto issue = [&](int g) {
#pragma unroll
      for (int t = 0; t < 2; t++) {
        const int c = lane + 32 * t, ck = c >> 4, cq = c & 15;
        const int64_t k = k0 + 4 * g + ck;
        const float *src = cq < 8 ? wp + k * a.Mp + cq * 4 : xp + k * a.Np + (cq - 8) * 4;
        cp_async16(ring + (g % NS) * STAGE + ck * ROW + cq * 4, src);
      }
    };
#pragma unroll
    for (int g = 0; g < NS - 1; g++) {
      if (g < groups) issue(g);
      cp_async_commit();
    }
    float2 acc[16];
#pragma unroll
    for (int i = 0; i < 16; i++) acc[i] = make_float2(0.0f, 0.0f);
    for (int g = 0; g < groups; g++) {
      cp_async_wait<NS - 2>();
      __syncwarp();  // every lane's copies of stage g landed; every lane is done with stage g - 1
      if (g + NS - 1 < groups) issue(g + NS - 1);
      cp_async_commit();
      const float *b = ring + (g % NS) * STAGE;
#pragma unroll
      for (int kk = 0; kk < 4; kk++) {
        const float4 w0 = *reinterpret_cast<const float4 *>(b + kk * ROW + mo);
        const float4 w1 = *reinterpret_cast<const float4 *>(b + kk * ROW + mo + 4);
        const float4 x4 = *reinterpret_cast<const float4 *>(b + kk * ROW + TM + ro);
        const float2 wq[4] = {make_float2(w0.x, w0.y), make_float2(w0.z, w0.w), make_float2(w1.x, w1.y),
                              make_float2(w1.z, w1.w)};
        const float xr[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const float2 xj = make_float2(xr[j], xr[j]);
#pragma unroll
          for (int i = 0; i < 4; i++) acc[j * 4 + i] = __ffma2_rn(wq[i], xj, acc[j * 4 + i]);
        }
      }
    }
    cp_async_wait<0>();
    __syncwarp();  // the ring is free for the next segment
#pragma unroll
    for (int i = 0; i < 16; i++) pair[i] = h == 0 ? acc[i] : __fadd2_rn(pair[i], acc[i]);
  }

  // The eight pair sums of each output, [warp][i][lane] (consecutive lanes,
  // consecutive float2), where the rings were.
  __syncthreads();
  float2 *red = reinterpret_cast<float2 *>(smem);
#pragma unroll
  for (int i = 0; i < 16; i++) red[(warp * 16 + i) * 32 + lane] = pair[i];
  __syncthreads();

  const int64_t rbase = (int64_t)bx * a.Nx;
#pragma unroll 1
  for (int u = 0; u < 2; u++) {
    const int q = threadIdx.x + u * THREADS;  // (i, l) = (q / 32, q % 32) of every warp's 512
    float2 p[8];
#pragma unroll
    for (int w = 0; w < 8; w++) p[w] = red[w * 512 + q];
    const float2 top = __fadd2_rn(__fadd2_rn(__fadd2_rn(p[0], p[1]), __fadd2_rn(p[2], p[3])),
                                  __fadd2_rn(__fadd2_rn(p[4], p[5]), __fadd2_rn(p[6], p[7])));
    const int i = q >> 5, l = q & 31;
    const int64_t rl = rl0 + (l >> 2) * 4 + (i >> 2);
    if (rl >= a.Nx) continue;
    const int64_t r = rbase + rl;
    const int mb = m0 + (l & 3) * 8 + 2 * (i & 3);
    float v[2] = {top.x, top.y};
#pragma unroll
    for (int e = 0; e < 2; e++) {
      const int m = mb + e;
      if (m >= a.M) continue;
      if (a.np < a.K) {
        const float *wr = a.w + (a.wbs ? (int64_t)bx * a.wbs : 0) + (int64_t)m * a.K;
        v[e] = dot_tail(wr, a.x + r * a.K, a.np, a.K, v[e], a.flavor);
      }
      v[e] = arm_nan(v[e]);
      if (EPI) {
        const float bb = (a.ep & EP_BIAS) ? __ldg(a.bias + m) : 0.0f;
        const float hh = (a.ep & EP_RES) ? __ldg(a.res + r * a.M + m) : 0.0f;
        v[e] = ep_add(a.ep, v[e], bb, hh);
      }
      a.y[r * a.M + m] = v[e];
    }
  }
}

void launch_mul_mat_seg(bool epi, unsigned grid, cudaStream_t stream, const MMArgs &a) {
  if (epi)
    k_mul_mat_seg<true><<<grid, sg::THREADS, 0, stream>>>(a);
  else
    k_mul_mat_seg<false><<<grid, sg::THREADS, 0, stream>>>(a);
}

}  // namespace shlo
