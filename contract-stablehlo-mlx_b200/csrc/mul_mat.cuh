// mul_mat's packed-segment kernels (ggml_vec_dot_f32 bit for bit): the shared
// definitions, the TMEM-stack kernel k_mul_mat_tm and the register-stack kernel
// k_mul_mat_short. The kernel instances are compiled in their own translation
// units (mul_mat_tm_split{1,2,4}.cu, mul_mat_short.cu), which define
// SHLO_MUL_MAT_INSTANCES; ggml_kernels.cu calls them through the launchers
// declared at the end.
#pragma once
#include <cuda.h>  // CUtensorMap (the type only; the encoder is reached through the runtime)

#include <utility>

#include "common.cuh"
#include "gelu.cuh"
#include "ggml_math.cuh"

namespace shlo {

// =============================================================== mul_mat ====
// y[r*M + m] = ggml_vec_dot_f32(w row (r/N)*wbs + m*K, x row r), K long
// (StablehloMlx/Kernels/Shaders.lean:55-91; Run.lean:64-65). ggml's order:
// sixteen accumulators a[j], j = k mod 16, each a k-ascending chain of fused
// multiply-adds starting at +0; the GGML_F32x4_REDUCE tree
// ((a0+a8)+(a4+a12)) + ((a1+a9)+(a5+a13)) + ((a2+a10)+(a6+a14)) + ((a3+a11)+(a7+a15))
// grouped as (v0+v1)+(v2+v3); then the tail of K mod 16 elements.
//
// The tree is a perfect binary tree whose leaves, left to right, are the
// classes 0, 8, 4, 12, 1, 9, 5, 13, 2, 10, 6, 14, 3, 11, 7, 15: class j is
// leaf 4*(j & 3) + r(j >> 2), with r the 2-bit reversal. The fast path packs
// each operand k-major with its K reordered so that leaf s's class fills the
// s-th contiguous segment of the packed K axis. Each class chain is then an
// ordinary k-ascending register-tiled GEMM over one segment; at each segment
// boundary the running accumulators fold into a four-level stack by the
// post-order of the tree (the binary-counter rule below), which adds exactly
// the same pairs in the same roles as ggml.
//
// Segments are padded to a multiple of 4 k-steps with w = -0 and x = +0: the
// product is -0 and acc + (-0) == acc for every acc (+0 stays +0, -0 stays -0),
// so padding leaves every chain bit-identical.

// The leaf of class j in the reduction tree.
__host__ __device__ constexpr int leaf_of_class(int j) {
  return 4 * (j & 3) + (((j >> 2) & 1) << 1 | ((j >> 3) & 1));
}
static_assert(leaf_of_class(0) == 0 && leaf_of_class(8) == 1 && leaf_of_class(4) == 2 && leaf_of_class(12) == 3 &&
                  leaf_of_class(1) == 4 && leaf_of_class(9) == 5 && leaf_of_class(5) == 6 &&
                  leaf_of_class(13) == 7 && leaf_of_class(2) == 8 && leaf_of_class(15) == 15,
              "ggml_vec_dot_f32 reduction-tree leaf order");

// One output, the reference's one-thread-per-output form; also the planted
// `plain` fault (a sequential binary32 sum without fma, Shaders.lean:65-68).
__device__ __forceinline__ float dot_tail(const float *w, const float *x, int np, int K, float sumf, int flavor) {
  int tl = K - np;
  if (flavor == 0) {  // pinned: separate product and sum
    for (int i = np; i < K; i++) sumf = __fadd_rn(sumf, __fmul_rn(w[i], x[i]));
  } else {  // stock: clang's form (Shaders.lean:80-90)
    int nq = tl >= 4 ? (tl & ~3) : 0;
    for (int i = np; i < np + nq; i++) sumf = __fadd_rn(sumf, __fmul_rn(w[i], x[i]));
    for (int i = np + nq; i < K; i++) sumf = __fmaf_rn(w[i], x[i], sumf);
  }
  return sumf;
}

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
  uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// mbarriers and TMA tile copies (k_mul_mat_tm's stage pipeline).
__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t *b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *b, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return done != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;\n" : "=l"(t));
  return t;
}
// Wait for the phase of parity `parity` of barrier b, for at most about two
// seconds, or until *abort is set (by another thread that gave up): false then.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *b, uint32_t parity, volatile int *abort) {
  if (mbar_try_wait(b, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1;; i++) {
    if (mbar_try_wait(b, parity)) return true;
    if ((i & 255) == 0 && (*abort || global_ns() - t0 > 2000000000ull)) return false;
  }
}
// A 2-D tile of the tensor map to shared memory, completing on barrier b.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *b) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(b))
      : "memory");
}


// Invalidate the L2 lines of n floats at p (a multiple of 32 floats from a
// 128-byte boundary) without writing them back: for scratch that was written
// and read within one launch and is never read again. The CTA's threads share
// the lines; call after every thread's last read of them.
__device__ __forceinline__ void discard_l2(float *p, size_t n) {
  for (size_t l = threadIdx.x; l < n / 32; l += blockDim.x)
    asm volatile("discard.global.L2 [%0], 128;\n" ::"l"(p + 32 * l) : "memory");
}

struct MMArgs {
  const float *wp;  // packed w [Wb][Kq][Mp]
  const float *xp;  // packed x [Bx][Kq][Np]
  const float *w;   // original w, for the tail
  const float *x;   // original x, for the tail
  float *y;
  int K, M, np, segp, Mp, Np;
  int64_t Nx;       // x rows per batch
  int64_t wbs;      // w batch stride (elements of the original w), 0 = shared
  int r_tiles;      // r tiles per batch
  int bx_count;     // x batches (1 when w is shared)
  int flavor;
  float *park;      // k_mul_mat_tm: 64 floats a thread a CTA, T(0..7) between the halves
  // Fused epilogue (the executor's bias and residual adds, each its own
  // binary32 rounding, in the module's operand order): EP_* flags.
  const float *bias;  // [M]
  const float *res;   // [R][M]
  int ep;
  int *ctr;           // k_mul_mat_tm split over CTAs: arrivals per tile (0 between launches)
  int *err;           // k_mul_mat_tm: set when a stage's copies did not arrive within the wait limit
  // k_mul_mat_tm with the gelu epilogue: ypk_np > 0 writes y as the packed x
  // of a next product whose K is M (segments of ypk_segp packed k, ypk_np
  // rows; (r, m) at (leaf_of_class(m % 16) * ypk_segp + m / 16) * ypk_np + r).
  int ypk_segp, ypk_np;
};


// y (the dot product, NaN already canonical) + bias[m], then + res[r][m]: the
// same __fadd_rn the built-in add runs, in the same operand order.
__device__ __forceinline__ float epilogue_adds(const MMArgs &a, float v, int64_t r, int m) {
  if (a.ep & EP_BIAS) {
    const float b = __ldg(a.bias + m);
    v = (a.ep & EP_BIAS_LHS) ? __fadd_rn(b, v) : __fadd_rn(v, b);
  }
  if (a.ep & EP_RES) {
    const float h = __ldg(a.res + r * a.M + m);
    v = (a.ep & EP_RES_LHS) ? __fadd_rn(h, v) : __fadd_rn(v, h);
  }
  return v;
}

// The epilogue operands of four outputs (r, mb..mb+3): 16-byte loads when M is
// a multiple of 4 and the four are in range, element loads otherwise.
__device__ __forceinline__ float4 ep_load4(const float *base, int64_t row, int mb, int M, bool vec) {
  const float *q = base + row * M + mb;
  if (vec && mb + 3 < M) return __ldg(reinterpret_cast<const float4 *>(q));
  float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  if (mb < M) v.x = __ldg(q);
  if (mb + 1 < M) v.y = __ldg(q + 1);
  if (mb + 2 < M) v.z = __ldg(q + 2);
  if (mb + 3 < M) v.w = __ldg(q + 3);
  return v;
}
__device__ __forceinline__ float ep_add(int ep, float v, float b, float h) {
  if (ep & EP_BIAS) v = (ep & EP_BIAS_LHS) ? __fadd_rn(b, v) : __fadd_rn(v, b);
  if (ep & EP_RES) v = (ep & EP_RES_LHS) ? __fadd_rn(h, v) : __fadd_rn(v, h);
  return v;
}

// ------------------------------------------------ the TMEM-stack mul_mat ----
// The same packed-segment algorithm with an 8 x 8 tile per thread (CTA tile
// 128 m x 128 r): the four stack levels of the reduction tree (64 values each per
// thread) live in Tensor Memory instead of registers. Warp w reaches TMEM lanes
// [32 (w % 4), +32); warps w and w + 4 share those lanes and split the 512
// columns: columns 256 (w / 4) + 64 L + [0, 64) hold level L. The stack is
// touched only at segment boundaries.
namespace mt {
// Two CTA shapes: WM = 2 warps along m gives a 128 m x 128 r tile, WM = 1 a
// 64 m x 256 r tile (for M <= 64, e.g. attention's value product).
constexpr int BK = 16, GPS = BK / 4, THREADS = 256;  // k per stage, groups of 4 k per stage
template <int WM>
struct Tile {
  static constexpr int BM = 64 * WM, BN = 256 / WM;
  static constexpr int STAGE_FLOATS = BK * (BM + BN);
};
// Two CTAs per SM (16 warps, 128 registers a thread). Each CTA holds 256 TMEM
// columns: stack levels 0 and 1 of its 8 warps (64 columns a level a warp).
// Level 2 (touched at 4 of 16 folds) is a 64 KB shared-memory slab; level 3
// (pushed once, at S = 7) is parked in a per-CTA global slice (it stays in L2)
// and added back in the epilogue.
constexpr int CTAS_PER_SM = 2;
constexpr int TMEM_COLS = 256;
constexpr int LEVEL_FLOATS = THREADS * 64;
template <int WM>
struct Pipe {
  static constexpr int NS = WM == 2 ? 3 : 2;  // stages of BK k
  // + 128: the stages start on a 128-byte boundary (TMA destinations)
  static constexpr size_t SMEM = (size_t)NS * Tile<WM>::STAGE_FLOATS * 4 + (size_t)LEVEL_FLOATS * 4 + 128;
  // A CTA that computes a quarter of the tree needs no level-2 slab: the same
  // shared memory holds more stages.
  static constexpr int NS_QUARTER = (int)((SMEM - 128) / (Tile<WM>::STAGE_FLOATS * 4));
};
// Dynamic shared memory above a third of an SM's: at most two CTAs per SM, so
// their TMEM columns (2 x 256) always fit the SM's 512.
static_assert(Pipe<2>::SMEM <= 113 * 1024 && Pipe<1>::SMEM <= 113 * 1024, "two CTAs per SM");
static_assert(3 * Pipe<2>::SMEM > 228 * 1024 && 3 * Pipe<1>::SMEM > 228 * 1024, "no third CTA on an SM");
}  // namespace mt

// 16 consecutive 32-bit TMEM columns of this thread's lane (32x32b shape: lane =
// the thread's lane in the warp's quarter), stored / loaded. Each waits for its
// own completion inside the same asm statement, so the registers are never used
// before they are valid.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float *v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};\n"
               "tcgen05.wait::st.sync.aligned;\n" ::"r"(taddr),
               "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
               "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
               "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
               "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
               "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
               "r"(__float_as_uint(v[15]))
               : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float *v) {
  uint32_t r[16];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];\n"
               "tcgen05.wait::ld.sync.aligned;\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                 "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
               : "r"(taddr)
               : "memory");
#pragma unroll
  for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

// 32 consecutive TMEM columns of this thread's lane, stored / loaded as one
// access with one wait (the fold moves two 16-column chunks at a time).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float *v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};\n"
      "tcgen05.wait::st.sync.aligned;\n" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])),
      "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
      "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])),
      "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float *v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

// Fold the finished chain of leaf S into the stack: pop and add the levels
// below the first zero bit of S (the left operand is the older value, as in the
// tree), then push at that level. Levels 0 and 1 are TMEM columns tcol + 64 L;
// level 2 is this thread's float4 slots of the shared-memory slab lv2, float4 j
// of chunk c at lv2[(c * 4 + j) * THREADS] (consecutive threads, consecutive
// float4: no bank conflicts). Level 3 is pushed only at S = 7 (depth 3) and
// popped only at S = 15 (depth 4); the caller parks it in global memory, so
// here depth 3 leaves the value in acc and depth 4 stops after level 2.
// PAIR: the adds as paired FP32 adds (fewer issue slots, more register pressure).
// last_pops >= 0: the last fold of a CTA that computes a subtree of 2^last_pops
// segments (a quarter: 2, an eighth: 1): pop that many levels, push nothing.
template <bool PAIR>
__device__ __forceinline__ void tfold_rt(float2 (&acc2)[32], uint32_t tcol, float4 *lv2, int S, int last_pops = -1) {
  const bool last = last_pops >= 0;
  const int depth = last ? last_pops : __ffs(~S) - 1;  // trailing one bits: 0..4
  const int pops = depth < 3 ? depth : 3;
  // Two chunks of 16 values at a time: 32 adjacent TMEM columns, one access.
#pragma unroll
  for (int cp = 0; cp < 2; cp++) {
    float v[32];
#pragma unroll
    for (int q = 0; q < 16; q++) {
      v[2 * q] = acc2[16 * cp + q].x;
      v[2 * q + 1] = acc2[16 * cp + q].y;
    }
    for (int L = 0; L < pops; L++) {
      float t[32];
      if (L < 2) {
        tmem_ld32(tcol + 64 * L + 32 * cp, t);
      } else {
#pragma unroll
        for (int j = 0; j < 8; j++) {
          const float4 u = lv2[(cp * 8 + j) * mt::THREADS];
          t[4 * j] = u.x; t[4 * j + 1] = u.y; t[4 * j + 2] = u.z; t[4 * j + 3] = u.w;
        }
      }
      if (PAIR) {
#pragma unroll
        for (int i = 0; i < 16; i++) {  // each component rounds as __fadd_rn
          const float2 r = __fadd2_rn(make_float2(t[2 * i], t[2 * i + 1]), make_float2(v[2 * i], v[2 * i + 1]));
          v[2 * i] = r.x;
          v[2 * i + 1] = r.y;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; i++) v[i] = __fadd_rn(t[i], v[i]);
      }
    }
    if (depth < 2 && !last) {
      tmem_st32(tcol + 64 * depth + 32 * cp, v);
    } else if (depth == 2 && !last) {
#pragma unroll
      for (int j = 0; j < 8; j++) lv2[(cp * 8 + j) * mt::THREADS] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    }
#pragma unroll
    for (int q = 0; q < 16; q++) acc2[16 * cp + q] = make_float2(v[2 * q], v[2 * q + 1]);
  }
}

// One CTA per tile, m-tile fastest (the CTAs running together share their x
// tile in L2).
// STAGE_FOLD: every segment spans whole stages (segp a multiple of 16), so the
// fold check runs once per stage; otherwise after every group of 4 k.
// SPLIT = 2, 4, 8 or 16: the grid has SPLIT CTAs a tile, CTA q computing the
// subtree of segments [q 16/SPLIT, (q + 1) 16/SPLIT) (1 segment: one chain, no
// stack; 2 or 4 segments: a 1- or 2-level stack, all in TMEM; 8: levels 0-1 in
// TMEM and 2 in the slab); each writes its partial to a per-tile slice of
// a.park, and the last of the tile's CTAs to arrive (an atomic count, no
// waiting) adds the top of ggml's tree over the SPLIT partials -- T0 + T1,
// ((T0 + T1) + (T2 + T3)), ... -- and runs the epilogue. More, shorter CTAs
// fill a grid that would leave SMs idle (small products: few rows or few
// tiles). SPLIT = 1: one CTA a tile, T(0..7) parked in a.park until the root
// add.
// EPI: 0 the plain product; 1 the fused bias / residual adds in the epilogue;
// 2 those adds and then gelu_erf (WM = 2), the tile passing through shared
// memory so that each warp finishes whole rows (separate instances, so the
// plain product compiles without them).
//
// The stages arrive by TMA: thread 0 copies stage st's w tile (BM x 16 k) and x
// tile (BN x 16 k) from the tensor maps tw, tx of the packed operands into slot
// st % NS, completing on the slot's full barrier; every warp waits on that
// barrier, reads the stage, and arrives on the slot's empty barrier; once all
// eight warps have, thread 0 refills the slot with stage st + NS. So no CTA-wide
// barrier runs in the k-loop (a warp runs ahead while its stages are in), and no
// thread computes copy addresses. Every wait is bounded: a stage that never
// arrives (about two seconds) sets *a.err, the CTA waits (bounded) for its own
// copies in flight, frees its TMEM and returns without writing.
template <int WM, bool STAGE_FOLD, int SPLIT, int EPI>
__global__ void __launch_bounds__(mt::THREADS, mt::CTAS_PER_SM)
    k_mul_mat_tm(MMArgs a, const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tx) {
  using namespace mt;
  constexpr int BM = Tile<WM>::BM, BN = Tile<WM>::BN, STAGE_FLOATS = Tile<WM>::STAGE_FLOATS;
  constexpr int SEGS = 16 / SPLIT;  // segments a CTA
  // At most 4 segments a CTA: a stack of levels 0-1 only (TMEM), so the level-2
  // slab's shared memory holds more stages.
  constexpr bool NO_SLAB = SPLIT >= 4;
  constexpr int LAST_POPS = SPLIT == 4 ? 2 : SPLIT == 8 ? 1 : -1;
  constexpr int NS = NO_SLAB ? Pipe<WM>::NS_QUARTER : Pipe<WM>::NS;
  extern __shared__ __align__(128) float smem_raw[];
  float *smem = reinterpret_cast<float *>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~(uintptr_t)127);
  __shared__ uint32_t tmem_base;
  __shared__ __align__(8) uint64_t full_bar[NS], empty_bar[NS];
  __shared__ int abort_flag;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Warps WM (m) x 8/WM (r), lanes 8 (m) x 4 (r); a thread's m are mo + [0,4)
  // and mo + 32 + [0,4), its r are ro + [0,4) and ro + 16 + [0,4).
  const int mo = (warp % WM) * 64 + (lane & 7) * 4;
  const int ro = (warp / WM) * 32 + (lane >> 3) * 4;
  // This CTA's tile: m0, batch bx, first row rl0 (recomputed where needed, so
  // nothing but the operand pointers stays live through the k-loop).
  auto pos = [&](int &m0, int &bx, int64_t &rl0) {
    const int mtiles = a.Mp / BM, tile = blockIdx.x / SPLIT;
    m0 = (tile % mtiles) * BM;
    bx = (tile / mtiles) / a.r_tiles;
    rl0 = (int64_t)((tile / mtiles) % a.r_tiles) * BN;
  };
  const int Kq = 16 * a.segp;
  // CTA q of a tile reads packed k rows [q SEGS segp, (q + 1) SEGS segp): the
  // tile's rows in the tensor maps (w [Wb Kq][Mp], x [Bx Kq][Np]).
  const int kq0 = (int)(blockIdx.x % SPLIT) * SEGS * a.segp;
  int tm0, wrow0, tr0, xrow0;
  {
    int m0, bx;
    int64_t rl0;
    pos(m0, bx, rl0);
    tm0 = m0;
    tr0 = (int)rl0;
    wrow0 = (a.wbs ? bx * Kq : 0) + kq0;
    xrow0 = bx * Kq + kq0;
  }
  const int nstages = Kq / SPLIT / BK;

  if (tid == 0) {
#pragma unroll
    for (int q = 0; q < NS; q++) {
      mbar_init(&full_bar[q], 1);
      mbar_init(&empty_bar[q], THREADS / 32);
    }
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
  }
  if (warp == 0) {
    uint32_t slot = (uint32_t)__cvta_generic_to_shared(&tmem_base);
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(slot),
                 "n"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;\n");
  const uint32_t tcol = tmem_base + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)(128 * (warp >> 2));

  // Thread 0's copies of stage st into slot q (both tiles on the slot's full
  // barrier, which then expects their bytes).
  auto issue = [&](int st, int q) {
    float *sb = smem + q * STAGE_FLOATS;
    mbar_expect_tx(&full_bar[q], STAGE_FLOATS * 4);
    tma_load_2d(sb, &tw, tm0, wrow0 + st * BK, &full_bar[q]);
    tma_load_2d(sb + BK * BM, &tx, tr0, xrow0 + st * BK, &full_bar[q]);
  };
  int nissued = 0;  // thread 0's count of stages copied
  if (tid == 0) {
    asm volatile("prefetch.tensormap [%0];\n" ::"l"(&tw) : "memory");
    asm volatile("prefetch.tensormap [%0];\n" ::"l"(&tx) : "memory");
    for (; nissued < NS && nissued < nstages; nissued++) issue(nissued, nissued);
  }

  // acc[j][i] (r index j, m index i) lives in pairs along m: acc2[4 j + i / 2].
  float2 acc2[32];
#pragma unroll
  for (int i = 0; i < 32; i++) acc2[i] = make_float2(0.0f, 0.0f);

  // T(0..7), the left half of the tree, waits in this CTA's slice of a.park
  // (float4 i of thread t at float4 index i * THREADS + t: coalesced).
  auto park = [&](bool load) {
    float4 *q = reinterpret_cast<float4 *>(a.park + (size_t)blockIdx.x * (THREADS * 64)) + tid;
#pragma unroll
    for (int i = 0; i < 16; i++) {
      float2 &p0 = acc2[2 * i], &p1 = acc2[2 * i + 1];
      if (load) {
        const float4 l3 = q[i * THREADS];
        p0 = __fadd2_rn(make_float2(l3.x, l3.y), p0);
        p1 = __fadd2_rn(make_float2(l3.z, l3.w), p1);
      } else {
        q[i * THREADS] = make_float4(p0.x, p0.y, p1.x, p1.y);
      }
    }
  };

  // Stage-major k-loop, the groups of 4 k of a stage unrolled; the chain of
  // segment S ends every segp/4 groups and folds into the stack (a runtime
  // depth: the number of trailing one bits of S).
  float4 *lv2 = reinterpret_cast<float4 *>(smem + NS * STAGE_FLOATS) + tid;
  int S = 0, gleft = a.segp / 4;
  auto fold_segment = [&]() {
    // A CTA of one segment has no stack: its chain is its partial.
    if constexpr (SPLIT < 16) tfold_rt<STAGE_FOLD>(acc2, tcol, lv2, S, (LAST_POPS >= 0 && S == SEGS - 1) ? LAST_POPS : -1);
    // After S = 7 the fold left T(0..7) in acc (depth 3 pushes nothing).
    if (SPLIT == 1 && S == 7) park(false);
    if (++S < SEGS) {
#pragma unroll
      for (int i = 0; i < 32; i++) acc2[i] = make_float2(0.0f, 0.0f);
    }
  };
  int slot = 0;        // stage st's slot, st % NS
  uint32_t phase = 0;  // the parity of st / NS
  int next_wait = 0;   // the first stage this thread has not yet waited for
  auto give_up = [&]() {
    abort_flag = 1;
    if (a.err) atomicExch(a.err, 1);
    return false;
  };
  // One stage: wait for its copies, run its 16 k (after each group of 4 k,
  // group_end()), release the slot, and (thread 0) refill it NS stages ahead.
  auto stage = [&](int st, auto group_end) -> bool {
    if (!mbar_wait_bounded(&full_bar[slot], phase, &abort_flag)) return give_up();
    __syncwarp();  // the lanes left their waits apart; the folds' tcgen05 accesses need the warp whole
    next_wait = st + 1;
    const float *ws = smem + slot * STAGE_FLOATS + mo;
    const float *xs = smem + slot * STAGE_FLOATS + BK * BM + ro;
#pragma unroll
    for (int q = 0; q < GPS; q++) {
#pragma unroll
      for (int kk = 0; kk < 4; kk++) {
        const float4 w0 = *reinterpret_cast<const float4 *>(ws + (4 * q + kk) * BM);
        const float4 w1 = *reinterpret_cast<const float4 *>(ws + (4 * q + kk) * BM + 32);
        const float4 x0 = *reinterpret_cast<const float4 *>(xs + (4 * q + kk) * BN);
        const float4 x1 = *reinterpret_cast<const float4 *>(xs + (4 * q + kk) * BN + 16);
        // Paired FP32 FMAs: each component rounds exactly as __fmaf_rn.
        const float2 wp2[4] = {make_float2(w0.x, w0.y), make_float2(w0.z, w0.w), make_float2(w1.x, w1.y),
                               make_float2(w1.z, w1.w)};
        const float xr[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
        for (int j = 0; j < 8; j++) {
          const float2 xj = make_float2(xr[j], xr[j]);
#pragma unroll
          for (int i = 0; i < 4; i++) acc2[j * 4 + i] = __ffma2_rn(wp2[i], xj, acc2[j * 4 + i]);
        }
      }
      group_end();
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[slot]);
    if (tid == 0 && st + NS < nstages) {
      if (!mbar_wait_bounded(&empty_bar[slot], phase, &abort_flag)) return give_up();
      issue(st + NS, slot);
      nissued++;
    }
    __syncwarp();
    if (++slot == NS) {
      slot = 0;
      phase ^= 1;
    }
    return true;
  };
  bool ok = true;
  if constexpr (STAGE_FOLD) {
    // Segments of whole stages: the fold between the segments' stage loops.
    const int sps = a.segp / BK;
    for (int st = 0; ok && S < SEGS;) {
      for (int e = st + sps; ok && st < e; st++) ok = stage(st, [] {});
      if (ok) fold_segment();
    }
  } else {
    for (int st = 0; ok && st < nstages; st++)
      ok = stage(st, [&] {
        if (--gleft == 0) {
          gleft = a.segp / 4;
          fold_segment();
        }
      });
  }
  if (!ok && tid == 0) {
    // Gave up: wait (bounded) for this CTA's copies still in flight before its
    // shared memory is released.
    __shared__ int never;
    never = 0;
    for (int q = next_wait; q < nissued; q++) mbar_wait_bounded(&full_bar[q % NS], (q / NS) & 1, &never);
  }

  // Every TMEM access of this CTA is complete (each waited): free the columns.
  asm volatile("tcgen05.fence::before_thread_sync;\n");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;\n");
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem_base), "n"(TMEM_COLS));
  if (abort_flag) return;  // read after the barrier: the same for every thread

  if (SPLIT > 1) {
    // This CTA's subtree to its slice; the last of the tile's CTAs adds the top
    // of the tree.
    __shared__ int last;
    const int tile = blockIdx.x / SPLIT;
    float4 *mine = reinterpret_cast<float4 *>(a.park + (size_t)blockIdx.x * (THREADS * 64)) + tid;
#pragma unroll
    for (int i = 0; i < 16; i++) mine[i * THREADS] = make_float4(acc2[2 * i].x, acc2[2 * i].y, acc2[2 * i + 1].x, acc2[2 * i + 1].y);
    __threadfence();
    __syncthreads();
    if (tid == 0) last = atomicAdd(a.ctr + tile, 1) == SPLIT - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (tid == 0) a.ctr[tile] = 0;  // ready for the next launch
    const float4 *base = reinterpret_cast<const float4 *>(a.park + (size_t)tile * SPLIT * (THREADS * 64)) + tid;
    auto add4 = [](float4 u, float4 v) {
      const float2 lo = __fadd2_rn(make_float2(u.x, u.y), make_float2(v.x, v.y));
      const float2 hi = __fadd2_rn(make_float2(u.z, u.w), make_float2(v.z, v.w));
      return make_float4(lo.x, lo.y, hi.x, hi.y);
    };
#pragma unroll
    for (int i = 0; i < 16; i++) {
      // every partial from L2 (this CTA's own too: it wrote it above), then the
      // top of the tree: neighbours first, as the perfect binary tree pairs them
      // (partial q pushes at level ctz(~q) after adding the levels below it,
      // the older value on the left: the binary-counter form of that tree)
      constexpr int TOP = SPLIT == 2 ? 1 : SPLIT == 4 ? 2 : SPLIT == 8 ? 3 : 4;
      float4 lv[TOP + 1];
#pragma unroll
      for (int q = 0; q < SPLIT; q++) {
        float4 v = __ldcg(base + q * 16 * THREADS + i * THREADS);
#pragma unroll
        for (int L = 0; L <= TOP; L++) {
          if (((q >> L) & 1) == 0 || L == TOP) {
            lv[L] = v;
            break;
          }
          v = add4(lv[L], v);
        }
      }
      acc2[2 * i] = make_float2(lv[TOP].x, lv[TOP].y);
      acc2[2 * i + 1] = make_float2(lv[TOP].z, lv[TOP].w);
    }
    // The partials are spent: drop their L2 lines instead of writing them back.
    __syncthreads();
    discard_l2(a.park + (size_t)tile * SPLIT * (THREADS * 64), SPLIT * THREADS * 64);
  } else {
    // The root of the tree: T(0..7) + T(8..15).
    park(true);
    // The parked slice is spent: drop its L2 lines instead of writing them back.
    __syncthreads();
    discard_l2(a.park + (size_t)blockIdx.x * (THREADS * 64), THREADS * 64);
  }
  // Epilogue: the tail (K mod 16 elements, in order) and the store.
  int m0, bx;
  int64_t rl0;
  pos(m0, bx, rl0);
  const int64_t rbase = (int64_t)bx * a.Nx;
  const bool vec = (a.M & 3) == 0;
  if constexpr (EPI == 2) {
    // The tile through shared memory (the stages and the slab are spent):
    // every thread stores its outputs (the tail added, NaN made arm64's), the
    // erf table is staged beside them, then warp w runs rows w, w + 8, ...:
    // lane l the outputs 4 l .. 4 l + 3, + bias (+ residual) in the module's
    // order and gelu_erf, loaded and stored as 16-byte vectors.
    static_assert(WM == 2 && BM == 128, "a row of the tile is 32 lanes x 4");
    constexpr int TS = BM + 4;  // a tile row: 16-byte aligned, rows 4 banks apart
    static_assert((size_t)BN * TS * 4 + sizeof(shlo_erf::ErfSmem) <= Pipe<WM>::SMEM - 128, "tile and table fit");
    float *tile = smem;
    shlo_erf::ErfSmem *tab = reinterpret_cast<shlo_erf::ErfSmem *>(smem + BN * TS);
    __syncthreads();  // every read of the slab is done
    shlo_erf::erf_smem_load(tab);
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int rr = ro + (j & 3) + (j >> 2) * 16;
      const int64_t r = rbase + rl0 + rr;
#pragma unroll
      for (int h = 0; h < 2; h++) {
        float v[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const float2 pr = acc2[j * 4 + 2 * h + (i >> 1)];
          v[i] = (i & 1) ? pr.y : pr.x;
          const int m = m0 + mo + 32 * h + i;
          if (a.np < a.K && m < a.M && rl0 + rr < a.Nx) {
            const float *wr = a.w + (a.wbs ? (int64_t)bx * a.wbs : 0) + (int64_t)m * a.K;
            v[i] = dot_tail(wr, a.x + r * a.K, a.np, a.K, v[i], a.flavor);
          }
          v[i] = arm_nan(v[i]);
        }
        *reinterpret_cast<float4 *>(tile + rr * TS + mo + 32 * h) = make_float4(v[0], v[1], v[2], v[3]);
      }
    }
    __syncthreads();
    const int mb = m0 + 4 * lane;
    const float4 bv = (a.ep & EP_BIAS) ? ep_load4(a.bias, 0, mb, a.M, vec) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (int rr = warp; rr < BN && rl0 + rr < a.Nx; rr += THREADS / 32) {
      const int64_t r = rbase + rl0 + rr;
      const float4 t = *reinterpret_cast<const float4 *>(tile + rr * TS + 4 * lane);
      const float4 hv = (a.ep & EP_RES) ? ep_load4(a.res, r, mb, a.M, vec) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      const float4 g = gelu4(make_float4(ep_add(a.ep, t.x, bv.x, hv.x), ep_add(a.ep, t.y, bv.y, hv.y),
                                         ep_add(a.ep, t.z, bv.z, hv.z), ep_add(a.ep, t.w, bv.w, hv.w)),
                             tab);
      if (a.ypk_np) {
        // back into the tile (this thread's own four values), stored packed below
        *reinterpret_cast<float4 *>(tile + rr * TS + 4 * lane) = g;
      } else if (vec && mb + 3 < a.M) {
        *reinterpret_cast<float4 *>(a.y + r * a.M + mb) = g;
      } else {
        const float gs[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
        for (int i = 0; i < 4; i++)
          if (mb + i < a.M) a.y[r * a.M + mb + i] = gs[i];
      }
    }
    if (a.ypk_np) {
      // The next product's packed x, a column of the tile at a time: warp w
      // the columns w, w + 8, ...; lane l the rows l, l + 32, ... (128-byte
      // stores). Rows past the operand's are zero, as the pack writes them.
      __syncthreads();
      for (int mm = warp; mm < BM && m0 + mm < a.M; mm += THREADS / 32) {
        const int m = m0 + mm;
        float *col = a.y + ((int64_t)leaf_of_class(m & 15) * a.ypk_segp + (m >> 4)) * a.ypk_np;
#pragma unroll
        for (int rr = lane; rr < BN; rr += 32)
          if (rl0 + rr < a.ypk_np) col[rl0 + rr] = rl0 + rr < a.Nx ? tile[rr * TS + mm] : 0.0f;
      }
    }
    return;
  }
  if constexpr (EPI == 1) {
    // Per half h: the bias and all eight rows' residuals loaded first (one
    // round trip), then the adds and the stores.
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const int mb = m0 + mo + 32 * h;
      const float4 bv = (a.ep & EP_BIAS) ? ep_load4(a.bias, 0, mb, a.M, vec) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      float4 rv[8];
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const int64_t rl = rl0 + ro + (j & 3) + (j >> 2) * 16;
        rv[j] = (a.ep & EP_RES) && rl < a.Nx ? ep_load4(a.res, rbase + rl, mb, a.M, vec) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      }
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const int64_t rl = rl0 + ro + (j & 3) + (j >> 2) * 16;
        if (rl >= a.Nx) continue;
        const int64_t r = rbase + rl;
        const float bs[4] = {bv.x, bv.y, bv.z, bv.w}, hs[4] = {rv[j].x, rv[j].y, rv[j].z, rv[j].w};
        float v[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const float2 pr = acc2[j * 4 + 2 * h + (i >> 1)];
          v[i] = (i & 1) ? pr.y : pr.x;
          const int m = mb + i;
          if (a.np < a.K && m < a.M) {
            const float *wr = a.w + (a.wbs ? (int64_t)bx * a.wbs : 0) + (int64_t)m * a.K;
            v[i] = dot_tail(wr, a.x + r * a.K, a.np, a.K, v[i], a.flavor);
          }
          v[i] = ep_add(a.ep, arm_nan(v[i]), bs[i], hs[i]);
        }
        if (vec && mb + 3 < a.M) {
          *reinterpret_cast<float4 *>(a.y + r * a.M + mb) = make_float4(v[0], v[1], v[2], v[3]);
        } else {
#pragma unroll
          for (int i = 0; i < 4; i++)
            if (mb + i < a.M) a.y[r * a.M + mb + i] = v[i];
        }
      }
    }
    return;
  }
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int64_t rl = rl0 + ro + (j & 3) + (j >> 2) * 16;
    if (rl >= a.Nx) continue;
    const int64_t r = rbase + rl;
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const int mb = m0 + mo + 32 * h;
      float v[4];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const float2 pr = acc2[j * 4 + 2 * h + (i >> 1)];
        v[i] = (i & 1) ? pr.y : pr.x;
        const int m = mb + i;
        if (a.np < a.K && m < a.M) {
          const float *wr = a.w + (a.wbs ? (int64_t)bx * a.wbs : 0) + (int64_t)m * a.K;
          v[i] = dot_tail(wr, a.x + r * a.K, a.np, a.K, v[i], a.flavor);
        }
        v[i] = arm_nan(v[i]);
      }
      if (vec && mb + 3 < a.M) {
        *reinterpret_cast<float4 *>(a.y + r * a.M + mb) = make_float4(v[0], v[1], v[2], v[3]);
      } else {
#pragma unroll
        for (int i = 0; i < 4; i++)
          if (mb + i < a.M) a.y[r * a.M + mb + i] = v[i];
      }
    }
  }
}

// Short K (segp == 4, K < 80: every segment is 4 packed k-steps, e.g.
// attention's K = 64 head dimension). The whole packed K of a 64 m x 64 r tile
// sits in shared memory (2 x 16 KB), each thread owns 4 m x 4 r outputs, and
// the 16 segments are unrolled with their folds known at compile time, so the
// 4-level stack lives in registers: no TMEM, and no fold waits. A thread's m
// are mo + [0,4), its r are ro + [0,4) (warps 2 (m) x 4 (r), lanes 8 x 4).
namespace ms {
constexpr int BM = 64, BN = 64, THREADS = 256;
}

template <int S>
__device__ __forceinline__ void fold_regs(float2 (&acc)[8], float2 (&st)[4][8]) {
  constexpr int depth = S == 15 ? 4 : (S & 1) == 0 ? 0 : (S & 3) == 1 ? 1 : (S & 7) == 3 ? 2 : 3;
#pragma unroll
  for (int L = 0; L < depth; L++)
#pragma unroll
    for (int i = 0; i < 8; i++) acc[i] = __fadd2_rn(st[L][i], acc[i]);
  if (depth < 4) {
#pragma unroll
    for (int i = 0; i < 8; i++) st[depth][i] = acc[i];
  }
}

template <int S, int NG>
__device__ __forceinline__ void seg_regs(const float *ws, const float *xs, float2 (&acc)[8], float2 (&st)[4][8]) {
  // ws, xs: this segment's 4 NG packed k rows (BM resp. BN wide)
#pragma unroll
  for (int i = 0; i < 8; i++) acc[i] = make_float2(0.0f, 0.0f);
#pragma unroll
  for (int kk = 0; kk < 4 * NG; kk++) {
    const float4 w4 = *reinterpret_cast<const float4 *>(ws + kk * ms::BM);
    const float4 x4 = *reinterpret_cast<const float4 *>(xs + kk * ms::BN);
    const float2 w01 = make_float2(w4.x, w4.y), w23 = make_float2(w4.z, w4.w);
    const float xr[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const float2 xj = make_float2(xr[j], xr[j]);
      acc[2 * j] = __ffma2_rn(w01, xj, acc[2 * j]);
      acc[2 * j + 1] = __ffma2_rn(w23, xj, acc[2 * j + 1]);
    }
  }
  fold_regs<S>(acc, st);
}

// NG groups of 4 k a segment. NG = 1: the whole packed K (64 rows) is loaded
// once; NG > 1: a ring of MS_NS one-segment stages.
constexpr int MS_NS = 4;
template <int NG>
struct ShortSmem {
  static constexpr int SEG = 4 * NG * (ms::BM + ms::BN);  // floats of one segment's stage
  static constexpr int FLOATS = NG == 1 ? 16 * SEG : MS_NS * SEG;
};

template <int NG, typename Issue, int... S>
__device__ __forceinline__ void all_segs(float *sm, int mo, int ro, float2 (&acc)[8], float2 (&st)[4][8], Issue issue,
                                         std::integer_sequence<int, S...>) {
  constexpr int SEG = ShortSmem<NG>::SEG;
  if constexpr (NG == 1) {
    (seg_regs<S, 1>(sm + S * SEG + mo, sm + S * SEG + 4 * ms::BM + ro, acc, st), ...);
  } else {
    auto one = [&](auto sc) {
      constexpr int s = decltype(sc)::value;
      cp_async_wait<MS_NS - 2>();
      __syncthreads();
      if (s + MS_NS - 1 < 16) issue(s + MS_NS - 1);
      cp_async_commit();
      float *b = sm + (s % MS_NS) * SEG;
      seg_regs<s, NG>(b + mo, b + 4 * NG * ms::BM + ro, acc, st);
    };
    (one(std::integral_constant<int, S>{}), ...);
  }
}

template <bool EPI, int NG>
__global__ void __launch_bounds__(ms::THREADS, 2) k_mul_mat_short(MMArgs a) {
  using namespace ms;
  constexpr int SEG = ShortSmem<NG>::SEG, KS = 4 * NG;  // packed k rows a segment
  __shared__ __align__(16) float sm[ShortSmem<NG>::FLOATS];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int mo = (warp & 1) * 32 + (lane & 7) * 4;
  const int ro = (warp >> 1) * 16 + (lane >> 3) * 4;
  const int mtiles = a.Mp / BM;
  const int m0 = (blockIdx.x % mtiles) * BM;
  const int rb = blockIdx.x / mtiles;
  const int bx = rb / a.r_tiles;
  const int64_t rl0 = (int64_t)(rb % a.r_tiles) * BN;
  const int64_t Kq = 16 * KS;
  const float *wp = a.wp + (a.wbs ? (int64_t)bx * Kq * a.Mp : 0) + m0;
  const float *xp = a.xp + (int64_t)bx * Kq * a.Np + rl0;
  // segment s's packed rows [s KS, (s + 1) KS) of w and x into buffer b
  auto copy_seg = [&](int s, float *b) {
#pragma unroll
    for (int i = 0; i < (KS * BM / 4 + THREADS - 1) / THREADS; i++) {
      const int q = tid + i * THREADS;
      if (q < KS * BM / 4) {
        const int row = q / (BM / 4), col = (q % (BM / 4)) * 4;
        cp_async16(b + row * BM + col, wp + (int64_t)(s * KS + row) * a.Mp + col);
        cp_async16(b + KS * BM + row * BN + col, xp + (int64_t)(s * KS + row) * a.Np + col);
      }
    }
  };
  if constexpr (NG == 1) {
    for (int s = 0; s < 16; s++) copy_seg(s, sm + s * SEG);
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
  } else {
#pragma unroll
    for (int s = 0; s < MS_NS - 1; s++) {
      copy_seg(s, sm + s * SEG);
      cp_async_commit();
    }
  }
  auto issue = [&](int s) { copy_seg(s, sm + (s % MS_NS) * SEG); };

  float2 acc[8], st[4][8];
  all_segs<NG>(sm, mo, ro, acc, st, issue, std::make_integer_sequence<int, 16>{});

  // Epilogue: the tail (K mod 16 elements, in order) and the store.
  const int64_t rbase = (int64_t)bx * a.Nx;
  const bool vec = (a.M & 3) == 0;
  const int mb = m0 + mo;
  float4 bv = make_float4(0.0f, 0.0f, 0.0f, 0.0f), rv[4];
  if (EPI) {  // the fused adds' operands, loaded before any is used
    if (a.ep & EP_BIAS) bv = ep_load4(a.bias, 0, mb, a.M, vec);
#pragma unroll
    for (int j = 0; j < 4; j++)
      rv[j] = (a.ep & EP_RES) && rl0 + ro + j < a.Nx ? ep_load4(a.res, rbase + rl0 + ro + j, mb, a.M, vec)
                                                      : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  }
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const int64_t rl = rl0 + ro + j;
    if (rl >= a.Nx) continue;
    const int64_t r = rbase + rl;
    float v[4] = {acc[2 * j].x, acc[2 * j].y, acc[2 * j + 1].x, acc[2 * j + 1].y};
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int m = mb + i;
      if (a.np < a.K && m < a.M) {
        const float *wr = a.w + (a.wbs ? (int64_t)bx * a.wbs : 0) + (int64_t)m * a.K;
        v[i] = dot_tail(wr, a.x + r * a.K, a.np, a.K, v[i], a.flavor);
      }
      v[i] = arm_nan(v[i]);
      if (EPI) {
        const float bs[4] = {bv.x, bv.y, bv.z, bv.w}, hs[4] = {rv[j].x, rv[j].y, rv[j].z, rv[j].w};
        v[i] = ep_add(a.ep, v[i], bs[i], hs[i]);
      }
    }
    if (vec && mb + 3 < a.M) {
      *reinterpret_cast<float4 *>(a.y + r * a.M + mb) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
#pragma unroll
      for (int i = 0; i < 4; i++)
        if (mb + i < a.M) a.y[r * a.M + mb + i] = v[i];
    }
  }
}


// ------------------------------------------------------------ launchers ----
// k_mul_mat_tm<WM, STAGE_FOLD, SPLIT, EPI> on `stream` (SPLIT CTAs a tile);
// the dynamic shared memory of each instance is raised first by
// mul_mat_tm_attributes<SPLIT>(). Errors are left for cudaGetLastError.
template <int SPLIT>
cudaError_t mul_mat_tm_attributes();
// tw, tx: the tensor maps of the packed w ([Wb Kq][Mp], box Tile<WM>::BM x 16)
// and x ([Bx Kq][Np], box Tile<WM>::BN x 16).
// epi: 0 the plain product, 1 the fused adds, 2 the adds and gelu_erf (WM = 2).
template <int SPLIT>
void launch_mul_mat_tm(int WM, bool stage_fold, int epi, unsigned grid, cudaStream_t stream, const MMArgs &a,
                       const CUtensorMap &tw, const CUtensorMap &tx);
// k_mul_mat_short<EPI, NG> with NG = ng (1..4).
void launch_mul_mat_short(int ng, bool epi, unsigned grid, cudaStream_t stream, const MMArgs &a);
// k_mul_mat_seg<EPI> (mul_mat_seg.cu): small products, 32 m x 32 r tiles.
namespace sg {
constexpr int TM = 32, TR = 32, THREADS = 256;
}
void launch_mul_mat_seg(bool epi, unsigned grid, cudaStream_t stream, const MMArgs &a);

#ifdef SHLO_MUL_MAT_INSTANCES
template <int SPLIT>
cudaError_t mul_mat_tm_attributes() {
  cudaError_t e = cudaSuccess;
  auto attr = [&](auto kern, size_t bytes) {
    if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  };
  attr(k_mul_mat_tm<1, false, SPLIT, 0>, mt::Pipe<1>::SMEM);
  attr(k_mul_mat_tm<1, false, SPLIT, 1>, mt::Pipe<1>::SMEM);
  attr(k_mul_mat_tm<1, true, SPLIT, 0>, mt::Pipe<1>::SMEM);
  attr(k_mul_mat_tm<1, true, SPLIT, 1>, mt::Pipe<1>::SMEM);
  attr(k_mul_mat_tm<2, false, SPLIT, 0>, mt::Pipe<2>::SMEM);
  attr(k_mul_mat_tm<2, false, SPLIT, 1>, mt::Pipe<2>::SMEM);
  attr(k_mul_mat_tm<2, false, SPLIT, 2>, mt::Pipe<2>::SMEM);
  attr(k_mul_mat_tm<2, true, SPLIT, 0>, mt::Pipe<2>::SMEM);
  attr(k_mul_mat_tm<2, true, SPLIT, 1>, mt::Pipe<2>::SMEM);
  attr(k_mul_mat_tm<2, true, SPLIT, 2>, mt::Pipe<2>::SMEM);
  return e;
}

template <int SPLIT>
void launch_mul_mat_tm(int WM, bool stage_fold, int epi, unsigned grid, cudaStream_t stream, const MMArgs &a,
                       const CUtensorMap &tw, const CUtensorMap &tx) {
  const size_t smem = WM == 1 ? mt::Pipe<1>::SMEM : mt::Pipe<2>::SMEM;
#define SHLO_TM(WMv, SF, E) k_mul_mat_tm<WMv, SF, SPLIT, E><<<grid, mt::THREADS, smem, stream>>>(a, tw, tx)
  if (WM == 1) {
    if (stage_fold) (epi ? SHLO_TM(1, true, 1) : SHLO_TM(1, true, 0));
    else (epi ? SHLO_TM(1, false, 1) : SHLO_TM(1, false, 0));
  } else if (epi == 2) {
    if (stage_fold) SHLO_TM(2, true, 2);
    else SHLO_TM(2, false, 2);
  } else {
    if (stage_fold) (epi ? SHLO_TM(2, true, 1) : SHLO_TM(2, true, 0));
    else (epi ? SHLO_TM(2, false, 1) : SHLO_TM(2, false, 0));
  }
#undef SHLO_TM
}
#endif

}  // namespace shlo
