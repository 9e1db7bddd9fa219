// Fused attention for the executor: ggml's scores (mul_mat over the head width),
// soft_max with its scale, and the value product (mul_mat over the keys) of one
// (batch, head) in one launch, every rounding of the three kernels kept
// (StablehloMlx/Kernels/Shaders.lean:55-123 for the two kernels; the module's
// dot_general / ggml.soft_max / dot_general / transpose chain, Lower.lean:157-182).
//
// One CTA of 8 warps per (batch, head, 32 queries), two CTAs an SM, so that one
// CTA's loads and soft_max overlap the other's products:
//   1. K (all S keys) and the CTA's 32 queries, loaded row-contiguously and
//      stored transposed into shared memory with the head width in ggml's
//      packed class-major order (K = 64: sixteen segments of 4);
//   2. the 32 x S scores with ggml_vec_dot_f32's chains and tree (S = 256:
//      8 keys x 4 queries a thread, the fold stack's levels 1-3 in TMEM;
//      S = 128: 4 x 4, the register-stack fold of k_mul_mat_short), NaN made
//      arm64's, into a row-major shared tile;
//   3. soft_max over each row exactly as g_soft_max (x * scale, the max,
//      ggml_v_expf(x - max), the four-lane group sums added in order to a
//      binary64 sum, y = e * (float)(1 / sum)), the rows held in registers so
//      that the probabilities can replace the scores in packed key order, while
//      V's rows are copied in;
//   4. the value product (S = 256: a pair of the 16 key segments a warp, 8 x 8
//      outputs a thread, the pairs' sums added up ggml's tree; S = 128: the
//      segments split over two halves of the CTA, 4 x 4 a thread, added as the
//      tree's root), written straight into the [B][S][H][64] layout of the
//      merged heads.
#include "common.cuh"
#include "ggml_math.cuh"
#include "mul_mat.cuh"

namespace shlo {

namespace at {
constexpr int DH = 64;        // head width: the scores' K
constexpr int NQ = 32;        // queries a CTA
constexpr int THREADS = 256;  // 8 warps
template <int S>
struct Smem {
  static constexpr int SW = S + 4;   // a score row (16-byte aligned, rows 4 banks apart)
  static constexpr int A = DH * S;   // K^T [64 packed d][S keys], then V [S packed keys][64 d]
  static constexpr int Q = DH * NQ;  // Q^T [64 packed d][32 queries], then the group sums, then partials
  static constexpr int SP = NQ * SW > S * NQ ? NQ * SW : S * NQ;  // scores [32][SW], then P [S packed keys][32]
  static constexpr size_t BYTES = (size_t)(A + Q + SP) * sizeof(float);
};
static_assert(Smem<256>::BYTES <= 113 * 1024, "two CTAs an SM");
}  // namespace at

struct AttnArgs {
  const float *q, *k, *v;
  int64_t qs[3], ks[3], vs[3];  // element strides of batch, position, head (the width is contiguous)
  float *o;                     // [B][S][H][64], or (ypk_np > 0) packed, see below
  int H;
  float sc;
  // S = 256, ypk_np > 0: o is written as the packed x of a next product whose K
  // is H * 64 (segments of ypk_segp packed k, ypk_np rows): (row r, column k) at
  // (leaf_of_class(k % 16) * ypk_segp + k / 16) * ypk_np + r, r = b S + s and
  // k = h 64 + d.
  int ypk_segp, ypk_np;
};

// Packed position of head-width index d (K = 64: segments of 4, no padding).
__device__ __forceinline__ constexpr int pk_d(int d) { return leaf_of_class(d & 15) * 4 + (d >> 4); }
// Packed position of key j for the value product (segments of S / 16).
template <int S>
__device__ __forceinline__ constexpr int pk_key(int j) { return leaf_of_class(j & 15) * (S / 16) + (j >> 4); }
// Shared-memory places. Each XORs the float4 group index of a column with a
// function of the row, so that the transposing stores spread over the banks
// while a thread's four consecutive columns stay one 16-byte vector.
template <int S>
__device__ __forceinline__ constexpr int k_at(int p, int key) {  // K^T
  return p * S + ((((key >> 2) ^ (p & 15)) << 2) | (key & 3));
}
__device__ __forceinline__ constexpr int q_at(int p, int q) {  // Q^T
  return p * at::NQ + ((((q >> 2) ^ (p & 7)) << 2) | (q & 3));
}
template <int S>
__device__ __forceinline__ constexpr int p_at(int p, int q) {  // P: the same for both halves of the value product
  return p * at::NQ + (((((q >> 2) ^ (p % (S / 16)) ^ ((p / (S / 16)) & 7))) & 7) << 2) + (q & 3);
}

// Score segment SG (packed d rows 4 SG .. 4 SG + 3): keys key..key+3 (w, m) by
// queries qr..qr+3 (x, r), then the fold into the register stack.
template <int SG, int S>
__device__ __forceinline__ void score_seg(const float *Ks, const float *Qs, int key, int qr, float2 (&acc)[8],
                                          float2 (&st)[4][8]) {
#pragma unroll
  for (int i = 0; i < 8; i++) acc[i] = make_float2(0.0f, 0.0f);
#pragma unroll
  for (int kk = 0; kk < 4; kk++) {
    const int p = 4 * SG + kk;
    const float4 w4 = *reinterpret_cast<const float4 *>(Ks + k_at<S>(p, key));
    const float4 x4 = *reinterpret_cast<const float4 *>(Qs + q_at(p, qr));
    const float2 w01 = make_float2(w4.x, w4.y), w23 = make_float2(w4.z, w4.w);
    const float xr[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const float2 xj = make_float2(xr[j], xr[j]);
      acc[2 * j] = __ffma2_rn(w01, xj, acc[2 * j]);
      acc[2 * j + 1] = __ffma2_rn(w23, xj, acc[2 * j + 1]);
    }
  }
  fold_regs<SG>(acc, st);
}

template <int S, int... SG>
__device__ __forceinline__ void score_segs(const float *Ks, const float *Qs, int key, int qr, float2 (&acc)[8],
                                           float2 (&st)[4][8], std::integer_sequence<int, SG...>) {
  (score_seg<SG, S>(Ks, Qs, key, qr, acc, st), ...);
}

// One pass of scores (S = 128: 4 keys x 4 queries a thread, the register stack
// of k_mul_mat_short): keys key..key+3 by queries qr..qr+3 into the score rows
// (NaN made arm64's). Not inlined, so that one pass's registers are all the
// compiler allocates for it.
template <int S>
__device__ __noinline__ void score_pass(const float *Ks, const float *Qs, float *Ss, int key, int qr) {
  float2 acc[8], st[4][8];
  score_segs<S>(Ks, Qs, key, qr, acc, st, std::make_integer_sequence<int, 16>{});
#pragma unroll
  for (int j = 0; j < 4; j++)
    *reinterpret_cast<float4 *>(Ss + (qr + j) * at::Smem<S>::SW + key) =
        make_float4(arm_nan(acc[2 * j].x), arm_nan(acc[2 * j].y), arm_nan(acc[2 * j + 1].x), arm_nan(acc[2 * j + 1].y));
}

// The scores' fold of segment S for a thread's 8 keys x 4 queries (16 paired
// accumulators): pop and add the levels below the first zero bit of S (the
// older value on the left, as in ggml's tree), then push at that level; level 0
// in registers, levels 1, 2 and 3 in 32 TMEM columns each (tcol + 32 (L - 1)).
// S is known at compile time.
template <int S>
__device__ __forceinline__ void fold8(float2 (&acc)[16], float2 (&st0)[16], uint32_t tcol) {
  constexpr int depth = S == 15 ? 4 : (S & 1) == 0 ? 0 : (S & 3) == 1 ? 1 : (S & 7) == 3 ? 2 : 3;
#pragma unroll
  for (int L = 0; L < depth; L++) {
    if (L == 0) {
#pragma unroll
      for (int i = 0; i < 16; i++) acc[i] = __fadd2_rn(st0[i], acc[i]);
    } else {
      float t[32];
      tmem_ld32(tcol + 32u * (uint32_t)(L - 1), t);
#pragma unroll
      for (int i = 0; i < 16; i++) acc[i] = __fadd2_rn(make_float2(t[2 * i], t[2 * i + 1]), acc[i]);
    }
  }
  if constexpr (depth == 0) {
#pragma unroll
    for (int i = 0; i < 16; i++) st0[i] = acc[i];
  } else if constexpr (depth < 4) {
    float v[32];
#pragma unroll
    for (int i = 0; i < 16; i++) {
      v[2 * i] = acc[i].x;
      v[2 * i + 1] = acc[i].y;
    }
    tmem_st32(tcol + 32u * (uint32_t)(depth - 1), v);
  }
}

// Score segment SG (packed d rows 4 SG .. 4 SG + 3): keys key..key+3 and
// key+32..key+35 (w, m) by queries qr..qr+3 (x, r), then the fold.
template <int SG, int S>
__device__ __forceinline__ void score_seg8(const float *Ks, const float *Qs, int key, int qr, float2 (&acc)[16],
                                           float2 (&st)[16], uint32_t tcol) {
#pragma unroll
  for (int i = 0; i < 16; i++) acc[i] = make_float2(0.0f, 0.0f);
#pragma unroll
  for (int kk = 0; kk < 4; kk++) {
    const int p = 4 * SG + kk;
    const float4 w0 = *reinterpret_cast<const float4 *>(Ks + k_at<S>(p, key));
    const float4 w1 = *reinterpret_cast<const float4 *>(Ks + k_at<S>(p, key + 32));
    const float4 x4 = *reinterpret_cast<const float4 *>(Qs + q_at(p, qr));
    const float2 wp2[4] = {make_float2(w0.x, w0.y), make_float2(w0.z, w0.w), make_float2(w1.x, w1.y),
                           make_float2(w1.z, w1.w)};
    const float xr[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const float2 xj = make_float2(xr[j], xr[j]);
#pragma unroll
      for (int i = 0; i < 4; i++) acc[4 * j + i] = __ffma2_rn(wp2[i], xj, acc[4 * j + i]);
    }
  }
  fold8<SG>(acc, st, tcol);
}

template <int S, int... SG>
__device__ __forceinline__ void score_segs8(const float *Ks, const float *Qs, int key, int qr, float2 (&acc)[16],
                                            float2 (&st)[16], uint32_t tcol, std::integer_sequence<int, SG...>) {
  (score_seg8<SG, S>(Ks, Qs, key, qr, acc, st, tcol), ...);
}

// The scores: keys key..key+3 and key+32..key+35 by queries qr..qr+3 into the
// score rows (NaN made arm64's). Not inlined, so that its registers are all the
// compiler allocates for it.
template <int S>
__device__ __noinline__ void score_pass8(const float *Ks, const float *Qs, float *Ss, int key, int qr, uint32_t tcol) {
  float2 acc[16], st[16];
  score_segs8<S>(Ks, Qs, key, qr, acc, st, tcol, std::make_integer_sequence<int, 16>{});
#pragma unroll
  for (int j = 0; j < 4; j++) {
#pragma unroll
    for (int h = 0; h < 2; h++)
      *reinterpret_cast<float4 *>(Ss + (qr + j) * at::Smem<S>::SW + key + 32 * h) =
          make_float4(arm_nan(acc[4 * j + 2 * h].x), arm_nan(acc[4 * j + 2 * h].y), arm_nan(acc[4 * j + 2 * h + 1].x),
                      arm_nan(acc[4 * j + 2 * h + 1].y));
  }
}

// Value segment SG of a half (its packed key rows SG S/16 .. of Vs and Ps,
// which point at the half's first row): head-width indices mo..mo+3 (w, m) by
// queries ro..ro+3 (x, r); the fold is the subtree's (SG = 0..7). Both halves
// run this one code, four k a trip.
template <int SG, int S>
__device__ __forceinline__ void value_seg(const float *Vs, const float *Ps, int mo, int ro, float2 (&acc)[8],
                                          float2 (&st)[4][8]) {
  constexpr int SEGK = S / 16;
#pragma unroll
  for (int i = 0; i < 8; i++) acc[i] = make_float2(0.0f, 0.0f);
#pragma unroll
  for (int kk = 0; kk < SEGK; kk++) {
    const int p = SG * SEGK + kk;
    const float4 w4 = *reinterpret_cast<const float4 *>(Vs + p * at::DH + mo);
    const float4 x4 = *reinterpret_cast<const float4 *>(Ps + p_at<S>(p, ro));
    const float2 w01 = make_float2(w4.x, w4.y), w23 = make_float2(w4.z, w4.w);
    const float xr[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const float2 xj = make_float2(xr[j], xr[j]);
      acc[2 * j] = __ffma2_rn(w01, xj, acc[2 * j]);
      acc[2 * j + 1] = __ffma2_rn(w23, xj, acc[2 * j + 1]);
    }
  }
  fold_regs<SG>(acc, st);
}

template <int S, int... SG>
__device__ __forceinline__ void value_segs(const float *Vs, const float *Ps, int mo, int ro, float2 (&acc)[8],
                                           float2 (&st)[4][8], std::integer_sequence<int, SG...>) {
  (value_seg<SG, S>(Vs, Ps, mo, ro, acc, st), ...);
}

// Key segment 2 w + LF of warp w's pair (S = 256): head-width indices mo..mo+3
// and mo+32..mo+35 (w, m) by queries ro..ro+3 and ro+16..ro+19 (x, r), one
// chain per output from zero. vo: V's element for (the pair's first packed
// key row, mo). P's float4 group of (row p, queries q..q+3) is
// (q/4) ^ (p % 16) ^ (p/16 % 8) (p_at); on the pair's rows p = 32 w + 16 LF + kk
// that is ((q/4) ^ 2w ^ LF ^ kk) % 8. po: the pair's first row; bq4: 4 (the
// class of this thread's first queries on that row, (ro/4 ^ 2w) % 8); the
// second queries' class is the first's ^ 4.
template <int LF, int S>
__device__ __forceinline__ void value_leaf8(const float *A, const float *SP, int vo, int po, int bq4,
                                            float2 (&acc)[32]) {
  constexpr int SEGK = S / 16;
#pragma unroll
  for (int i = 0; i < 32; i++) acc[i] = make_float2(0.0f, 0.0f);
#pragma unroll
  for (int kk = 0; kk < SEGK; kk++) {
    const int r = LF * SEGK + kk;  // the row within the pair
    const int c4 = ((kk ^ LF) & 7) << 2;
    const float4 w0 = *reinterpret_cast<const float4 *>(A + vo + r * at::DH);
    const float4 w1 = *reinterpret_cast<const float4 *>(A + vo + r * at::DH + 32);
    const float4 x0 = *reinterpret_cast<const float4 *>(SP + po + (bq4 ^ c4) + r * at::NQ);
    const float4 x1 = *reinterpret_cast<const float4 *>(SP + po + (bq4 ^ c4 ^ 16) + r * at::NQ);
    const float2 wp2[4] = {make_float2(w0.x, w0.y), make_float2(w0.z, w0.w), make_float2(w1.x, w1.y),
                           make_float2(w1.z, w1.w)};
    const float xr[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const float2 xj = make_float2(xr[j], xr[j]);
#pragma unroll
      for (int i = 0; i < 4; i++) acc[4 * j + i] = __ffma2_rn(wp2[i], xj, acc[4 * j + i]);
    }
  }
}

// The value product's subtree of warp w (S = 256): T(2w) + T(2w + 1), the
// older on the left as in ggml's tree, left in this thread's 64 TMEM columns
// (tcol), where T(2w) waits for T(2w + 1). Not inlined, so that its registers
// are all the compiler allocates for it.
template <int S>
__device__ __noinline__ void value_pair8(const float *A, const float *SP, int warp, int mo, int ro, uint32_t tcol) {
  float2 acc[32];
  const int bq4 = (((ro >> 2) ^ (2 * warp)) & 7) << 2;
  const int po = warp * 32 * at::NQ;
  const int vo = warp * 32 * at::DH + mo;
  value_leaf8<0, S>(A, SP, vo, po, bq4, acc);
#pragma unroll
  for (int hf = 0; hf < 2; hf++) {
    float v[32];
#pragma unroll
    for (int i = 0; i < 16; i++) {
      v[2 * i] = acc[16 * hf + i].x;
      v[2 * i + 1] = acc[16 * hf + i].y;
    }
    tmem_st32(tcol + 32u * (uint32_t)hf, v);
  }
  value_leaf8<1, S>(A, SP, vo, po, bq4, acc);
#pragma unroll
  for (int hf = 0; hf < 2; hf++) {
    float t[32];
    tmem_ld32(tcol + 32u * (uint32_t)hf, t);
#pragma unroll
    for (int i = 0; i < 16; i++) {
      const float2 r = __fadd2_rn(make_float2(t[2 * i], t[2 * i + 1]), acc[16 * hf + i]);
      t[2 * i] = r.x;
      t[2 * i + 1] = r.y;
    }
    tmem_st32(tcol + 32u * (uint32_t)hf, t);
  }
}

template <int S>
__global__ void __launch_bounds__(at::THREADS, 2) k_attention(AttnArgs a) {
  using namespace at;
  using L = Smem<S>;
  extern __shared__ __align__(16) float sm[];
  float *A = sm, *Qs = sm + L::A, *SP = Qs + L::Q;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int NQB = S / NQ;
  const int qb = blockIdx.x % NQB, bh = blockIdx.x / NQB, h = bh % a.H, b = bh / a.H;
  const int i0 = qb * NQ;

  // 1. K and Q: sixteen lanes read a row's 256 bytes (two rows an instruction),
  //    every load in flight at once; lane l's four head-width floats 4 (l % 16)
  //    .. + 3 go to their packed rows.
  {
    constexpr int NR = (S + NQ) * 16 / THREADS;  // 16-byte loads a thread
    const int dc = tid & 15, r0 = tid >> 4;
    const float *kb = a.k + (int64_t)b * a.ks[0] + (int64_t)h * a.ks[2] + 4 * dc;
    const float *qbp = a.q + (int64_t)b * a.qs[0] + (int64_t)i0 * a.qs[1] + (int64_t)h * a.qs[2] + 4 * dc;
    float4 t[NR];
#pragma unroll
    for (int i = 0; i < NR; i++) {
      const int row = r0 + 16 * i;
      t[i] = __ldg(reinterpret_cast<const float4 *>(i < S / 16 ? kb + (int64_t)row * a.ks[1]
                                                               : qbp + (int64_t)(row - S) * a.qs[1]));
    }
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const int p = pk_d(4 * dc + e);
#pragma unroll
      for (int i = 0; i < NR; i++) {
        const int row = r0 + 16 * i;
        const float v = e == 0 ? t[i].x : e == 1 ? t[i].y : e == 2 ? t[i].z : t[i].w;
        if (i < S / 16) A[k_at<S>(p, row)] = v;
        else Qs[q_at(p, row - S)] = v;
      }
    }
  }
  __syncthreads();

  // 2. Scores: warps 4 (keys) x 2 (queries), lanes 8 (keys) x 4 (queries).
  //    S = 256: a thread 8 keys x 4 queries in one pass, levels 1 to 3 of the
  //    fold's stack in TMEM (256 columns a CTA, two CTAs an SM: warps w and
  //    w + 4 share lanes 32 (w % 4) .. + 32 and take columns 128 (w / 4) ..).
  //    S = 128: 4 keys x 4 queries, the whole stack in registers.
  __shared__ uint32_t tmem_base;
  uint32_t tcol = 0;
  if constexpr (S == 256) {
    if (warp == 0) {
      const uint32_t slot = (uint32_t)__cvta_generic_to_shared(&tmem_base);
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 256;\n" ::"r"(slot));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
    }
    asm volatile("tcgen05.fence::before_thread_sync;\n");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;\n");
    tcol = tmem_base + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)(128 * (warp >> 2));
    score_pass8<S>(A, Qs, SP, (warp & 3) * 64 + (lane & 7) * 4, (warp >> 2) * 16 + (lane >> 3) * 4, tcol);
    // (the columns stay allocated for the value product's fold)
    __syncthreads();
  } else {
    const int km = (warp & 3) * 32 + (lane & 7) * 4;
    const int qr = (warp >> 2) * 16 + (lane >> 3) * 4;
#pragma unroll 1
    for (int kb = 0; kb < S; kb += 128) score_pass<S>(A, Qs, SP, kb + km, qr);
    __syncthreads();
  }

  // 3. V's rows into A (now free) in packed key order, while soft_max runs.
  {
    const float *vb = a.v + (int64_t)b * a.vs[0] + (int64_t)h * a.vs[2];
#pragma unroll
    for (int i = 0; i < S * 16 / THREADS; i++) {
      const int c = tid + i * THREADS, j = c >> 4, dq = (c & 15) * 4;
      cp_async16(A + pk_key<S>(j) * DH + dq, vb + (int64_t)j * a.vs[1] + dq);
    }
    cp_async_commit();
  }
  // soft_max: warp w owns rows 4w..4w+3, eight lanes a row; lane g of a row
  // holds the four-key groups g, g + 8, g + 16, ... in registers.
  {
    constexpr int G = S / 32;  // groups a lane
    const int r = lane >> 3, g = lane & 7, q = 4 * warp + r;
    const float *row = SP + q * L::SW;
    float *parts = Qs + q * (S / 4);  // the row's group sums, in group order
    float4 e[G];
    float mx = -INFINITY;
    bool nan = false;
#pragma unroll
    for (int t = 0; t < G; t++) {
      float4 x = *reinterpret_cast<const float4 *>(row + 4 * (g + 8 * t));
      x.x = __fmul_rn(x.x, a.sc); x.y = __fmul_rn(x.y, a.sc); x.z = __fmul_rn(x.z, a.sc); x.w = __fmul_rn(x.w, a.sc);
      e[t] = x;
      nan |= (x.x != x.x) | (x.y != x.y) | (x.z != x.z) | (x.w != x.w);
      mx = fmaxf(mx, fmaxf(fmaxf(x.x, x.y), fmaxf(x.z, x.w)));
    }
    // The max of a row without NaN is order-free (which zero it is cannot
    // change an output); a row with a NaN takes the spec's sequential scan.
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const unsigned rowmask = 0xFFu << (8 * r);
    const bool row_nan = (__ballot_sync(0xffffffffu, nan) & rowmask) != 0;
    if (row_nan && g == 0) {
      float m = -INFINITY;
      for (int i = 0; i < S; i++) {
        const float wv = __fmul_rn(row[i], a.sc);
        m = (m > wv) ? m : wv;
      }
      mx = m;
    }
    mx = __shfl_sync(0xffffffffu, mx, 8 * r);
    int pmin = 255, pmax = 0;
    bool pspecial = false;
    double psum = 0.0;
#pragma unroll
    for (int t = 0; t < G; t++) {
      float4 y;
      y.x = ggml_v_expf(__fsub_rn(e[t].x, mx));
      y.y = ggml_v_expf(__fsub_rn(e[t].y, mx));
      y.z = ggml_v_expf(__fsub_rn(e[t].z, mx));
      y.w = ggml_v_expf(__fsub_rn(e[t].w, mx));
      e[t] = y;
      const float part = __fadd_rn(__fadd_rn(y.x, y.y), __fadd_rn(y.z, y.w));
      parts[g + 8 * t] = part;
      // the binades the row's group sums span (all positive or zero)
      const uint32_t pb = fbits(part) & 0x7FFFFFFFu;
      const int pe = (int)(pb >> 23);
      pspecial |= pe == 255;
      if (pb) {
        pmin = min(pmin, pe ? pe : 1);
        pmax = max(pmax, pe ? pe : 1);
      }
      psum = __dadd_rn(psum, (double)part);
    }
    // When the group sums' nonzero terms span few enough binades, every partial
    // sum of them is exact in binary64 (multiples of 2^(pmin - 150) below
    // 2^(pmax - 126 + log2(S / 4))), so the order of the adds cannot matter: the
    // row's eight lanes add their parts and a shuffle tree gives the spec's sum.
    // Otherwise one lane runs the spec's serial chain.
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) {
      pmin = min(pmin, __shfl_xor_sync(0xffffffffu, pmin, o));
      pmax = max(pmax, __shfl_xor_sync(0xffffffffu, pmax, o));
    }
    constexpr int LG = S == 256 ? 6 : 5;  // log2 of the group count
    const bool exact = (__ballot_sync(0xffffffffu, pspecial) & rowmask) == 0 && (pmin > pmax || pmax - pmin + 24 + LG <= 53);
    // Every lane takes part in the shuffles and the barrier (the four rows of a
    // warp may differ in `exact`); the branches below hold no warp collective.
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) psum = __dadd_rn(psum, __shfl_xor_sync(0xffffffffu, psum, o));
    __syncwarp();  // the parts, for the serial chain
    float inv = 0.0f;
    if (exact) {
      inv = __double2float_rn(__ddiv_rn(1.0, psum));
    } else if (g == 0) {
      double sum = 0.0;
      for (int k = 0; k < S / 4; k += 8) {  // eight parts loaded ahead of their serial adds
        double v[8];
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] = (double)parts[k + i];
#pragma unroll
        for (int i = 0; i < 8; i++) sum = __dadd_rn(sum, v[i]);
      }
      inv = __double2float_rn(__ddiv_rn(1.0, sum));
    }
    inv = __shfl_sync(0xffffffffu, inv, 8 * r);
    __syncthreads();  // every score read (the scans too): P may now replace them
    float *Ps = SP;
#pragma unroll
    for (int t = 0; t < G; t++) {
      const int j0 = 4 * (g + 8 * t);
      const float y[4] = {arm_nan(__fmul_rn(e[t].x, inv)), arm_nan(__fmul_rn(e[t].y, inv)),
                          arm_nan(__fmul_rn(e[t].z, inv)), arm_nan(__fmul_rn(e[t].w, inv))};
#pragma unroll
      for (int c = 0; c < 4; c++) Ps[p_at<S>(pk_key<S>(j0 + c), q)] = y[c];
    }
  }
  cp_async_wait<0>();
  __syncthreads();

  // 4. The value product. S = 256: warp w the key segments 2w and 2w + 1, a
  //    thread 8 head-width indices x 8 queries; then the subtrees' sums up
  //    ggml's tree through shared memory (V spent): warp 2i + 1 hands its tile
  //    to 2i, 4i + 2 to 4i, 4 to 0, each level in a region of its own, and
  //    warp 0 stores the root.
  if constexpr (S == 256) {
    const int mo = (lane & 7) * 4, ro = (lane >> 3) * 4;
    value_pair8<S>(A, SP, warp, mo, ro, tcol);
    float2 acc[32];
#pragma unroll
    for (int hf = 0; hf < 2; hf++) {
      float t[32];
      tmem_ld32(tcol + 32u * (uint32_t)hf, t);
#pragma unroll
      for (int i = 0; i < 16; i++) acc[16 * hf + i] = make_float2(t[2 * i], t[2 * i + 1]);
    }
    asm volatile("tcgen05.fence::before_thread_sync;\n");
    __syncthreads();  // every read of V and P and every TMEM access is done
    asm volatile("tcgen05.fence::after_thread_sync;\n");
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;\n" ::"r"(tmem_base));
    float4 *xch = reinterpret_cast<float4 *>(A) + lane;
#pragma unroll
    for (int lvl = 1; lvl <= 3; lvl++) {
      // level lvl: warps w with w % 2^(lvl-1) == 0 hold a subtree; the odd
      // ones among them (w / 2^(lvl-1) odd) hand it to w - 2^(lvl-1)
      const int base = lvl == 1 ? 0 : lvl == 2 ? 4 : 6;  // the level's first slot of 512 float4
      const bool holds = (warp & ((1 << (lvl - 1)) - 1)) == 0;
      const bool gives = holds && ((warp >> (lvl - 1)) & 1);
      float4 *slot = xch + (base + (warp >> lvl)) * 512;
      if (gives) {
#pragma unroll
        for (int i = 0; i < 16; i++) slot[32 * i] = make_float4(acc[2 * i].x, acc[2 * i].y, acc[2 * i + 1].x, acc[2 * i + 1].y);
      }
      __syncthreads();
      if (holds && !gives) {
#pragma unroll
        for (int i = 0; i < 16; i++) {
          const float4 u = slot[32 * i];
          acc[2 * i] = __fadd2_rn(acc[2 * i], make_float2(u.x, u.y));
          acc[2 * i + 1] = __fadd2_rn(acc[2 * i + 1], make_float2(u.z, u.w));
        }
      }
    }
    if (a.ypk_np) {
      // The packed layout: the root's tile through shared memory ([64 d][32
      // queries + 1] over the first level's slots, read before the second
      // level's barrier); then warp w the columns 8w .. 8w + 7, lane l query l
      // (128-byte stores).
      float *tt = A;
      if (warp == 0) {
#pragma unroll
        for (int j = 0; j < 8; j++) {
          const int q = ro + (j & 3) + (j >> 2) * 16;
#pragma unroll
          for (int i = 0; i < 4; i++) {
            const float2 pr = acc[4 * j + i];
            const int d = mo + (i & 1) * 2 + (i >> 1) * 32;
            tt[d * 33 + q] = arm_nan(pr.x);
            tt[(d + 1) * 33 + q] = arm_nan(pr.y);
          }
        }
      }
      __syncthreads();
#pragma unroll
      for (int c = 0; c < 8; c++) {
        const int d = 8 * warp + c, k = h * DH + d;
        a.o[((int64_t)leaf_of_class(k & 15) * a.ypk_segp + (k >> 4)) * a.ypk_np + (int64_t)b * S + i0 + lane] =
            tt[d * 33 + lane];
      }
    } else if (warp == 0) {
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const int q = ro + (j & 3) + (j >> 2) * 16;
        float *dst = a.o + (((int64_t)b * S + i0 + q) * a.H + h) * DH + mo;
#pragma unroll
        for (int hf = 0; hf < 2; hf++) {
          const float2 lo = acc[4 * j + 2 * hf], hi = acc[4 * j + 2 * hf + 1];
          *reinterpret_cast<float4 *>(dst + 32 * hf) = make_float4(arm_nan(lo.x), arm_nan(lo.y), arm_nan(hi.x), arm_nan(hi.y));
        }
      }
    }
  } else {
    // S = 128: warps 0-3 the segments 0-7 (T(0..7)), warps 4-7 the segments
    // 8-15 (T(8..15)); each half's warps 2 (width) x 2 (queries), 4 x 4 a thread.
    const int wg = warp & 3, half = warp >> 2;
    const int mo = (wg & 1) * 32 + (lane & 7) * 4;
    const int ro = (wg >> 1) * 16 + (lane >> 3) * 4;
    const int row0 = half * 8 * (S / 16);  // the half's first packed key row
    float2 acc[8], st[4][8];
    value_segs<S>(A + row0 * DH, SP + row0 * NQ, mo, ro, acc, st, std::make_integer_sequence<int, 8>{});
    float4 *part = reinterpret_cast<float4 *>(Qs) + (tid & 127);  // the group sums are spent
    if (half == 1) {
#pragma unroll
      for (int i = 0; i < 4; i++) part[i * 128] = make_float4(acc[2 * i].x, acc[2 * i].y, acc[2 * i + 1].x, acc[2 * i + 1].y);
    }
    __syncthreads();
    if (half == 0) {
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const float4 u = part[j * 128];
        const float2 lo = __fadd2_rn(acc[2 * j], make_float2(u.x, u.y));      // the root: T(0..7) + T(8..15)
        const float2 hi = __fadd2_rn(acc[2 * j + 1], make_float2(u.z, u.w));
        float *dst = a.o + (((int64_t)b * S + i0 + ro + j) * a.H + h) * DH + mo;
        *reinterpret_cast<float4 *>(dst) = make_float4(arm_nan(lo.x), arm_nan(lo.y), arm_nan(hi.x), arm_nan(hi.y));
      }
    }
  }
}

// q, k, v: [B][S][H][64] views (any element strides of the first three
// dimensions, the width contiguous); p = [B, S, H, width, scale bits].
int k_attention(Device *dev, Arr *q, Arr *k, Arr *v, const uint32_t *p, Arr **out) {
  return k_attention_packed(dev, q, k, v, p, nullptr, out);
}

int k_attention_packed(Device *dev, Arr *q, Arr *k, Arr *v, const uint32_t *p, const int *y_pack, Arr **out) {
  const int64_t B = p[0], S = p[1], H = p[2], W = p[3];
  const float sc = bitsf_host(p[4]);
  if (W != at::DH || (S != 128 && S != 256) || B <= 0 || H <= 0)
    return fail("attention: B=%lld S=%lld H=%lld width=%lld not carried (width 64, S 128 or 256)", (long long)B,
                (long long)S, (long long)H, (long long)W);
  Arr *in[3] = {q, k, v};
  Arr *own[3] = {nullptr, nullptr, nullptr};
  AttnArgs a{};
  int64_t *strides[3] = {a.qs, a.ks, a.vs};
  const float *ptrs[3];
  int rc = 0;
  for (int i = 0; i < 3 && !rc; i++) {
    Arr *x = in[i];
    if (x->dtype != kF32) {
      rc = fail("attention: input %d is %s, f32 expected", i, dtype_name(x->dtype));
      break;
    }
    if (x->ndim != 4 || x->shape[0] != B || x->shape[1] != S || x->shape[2] != H || x->shape[3] != W) {
      rc = fail("attention: input %d is not [%lld, %lld, %lld, %lld]", i, (long long)B, (long long)S, (long long)H,
                (long long)W);
      break;
    }
    // 16-byte rows: the width contiguous, every row start a multiple of 4 floats.
    bool ok = x->strides[3] == 1 && ((uintptr_t)data_ptr(x) & 15) == 0;
    for (int d = 0; d < 3; d++) ok = ok && x->strides[d] % 4 == 0;
    if (!ok) {
      if ((rc = make_contiguous(x, &own[i]))) break;
      x = own[i];
    }
    for (int d = 0; d < 3; d++) strides[i][d] = x->strides[d];
    ptrs[i] = (const float *)data_ptr(x);
  }
  Arr *o = nullptr;
  // the packed layout in the kernel's epilogue (S = 256, no padded rows), else
  // by the pack kernel after it
  const bool pk_epi = y_pack && S == 256 && y_pack[1] == B * S && 16 * (int64_t)y_pack[0] == H * W;
  if (!rc) {
    int64_t shape[1] = {pk_epi ? H * W * (int64_t)y_pack[1] : B * S * H * W};
    rc = new_array(dev, kF32, shape, 1, &o);
    if (!rc) o->shape[0] = B * S * H * W;
  }
  if (!rc) {
    a.q = ptrs[0];
    a.k = ptrs[1];
    a.v = ptrs[2];
    a.o = (float *)o->buf->ptr;
    a.H = (int)H;
    a.sc = sc;
    if (pk_epi) {
      a.ypk_segp = y_pack[0];
      a.ypk_np = y_pack[1];
    }
    static bool attr_done[64] = {false};
    if (!attr_done[dev->id]) {
      rc = cuda_check(cudaFuncSetAttribute(k_attention<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)at::Smem<128>::BYTES), "attention attribute") ||
           cuda_check(cudaFuncSetAttribute(k_attention<256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)at::Smem<256>::BYTES), "attention attribute");
      if (!rc) attr_done[dev->id] = true;
    }
  }
  if (!rc) {
    const unsigned grid = (unsigned)(B * H * (S / at::NQ));
    if (S == 256)
      k_attention<256><<<grid, at::THREADS, at::Smem<256>::BYTES, dev->stream>>>(a);
    else
      k_attention<128><<<grid, at::THREADS, at::Smem<128>::BYTES, dev->stream>>>(a);
    rc = launch_check("attention");
  }
  for (int i = 0; i < 3; i++)
    if (own[i]) shlo_release(own[i]);
  if (!rc && y_pack && !pk_epi) {
    Arr *pk;
    rc = k_pack_x(dev, o, B * S, H * W, y_pack, &pk);
    shlo_release(o);
    o = rc ? nullptr : pk;
  }
  if (rc) {
    if (o) shlo_release(o);
    return 1;
  }
  *out = o;
  return 0;
}

}  // namespace shlo
