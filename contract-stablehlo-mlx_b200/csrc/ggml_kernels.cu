// The exact kernels: ggml-cpu's arm64 arithmetic, bit for bit, on sm_100a.
//
// Each kernel reproduces the reference's Lean kernel spec
// (StablehloMlx/Kernels/Shaders.lean) with the parameter words of
// StablehloMlx/Kernels/Run.lean:62-104. Built with -fmad=false: every fused
// multiply-add below is an explicit __fmaf_rn where ggml uses vfmaq_f32, and
// every other product and sum is rounded on its own.
#include <cmath>

#include "common.cuh"
#include <utility>

#include "erff_cr.cuh"

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

static int check_elems(Arr *a, int64_t need, const char *what) {
  if (numel(a) < need)
    return fail("%s: input of %lld elements, the parameters need %lld", what, (long long)numel(a), (long long)need);
  return 0;
}

static int require_dtype(Arr *a, int dt, const char *what) {
  if (a->dtype != dt) return fail("%s: input is %s, %s expected", what, dtype_name(a->dtype), dtype_name(dt));
  return 0;
}

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

__global__ void k_mul_mat_naive(const float *__restrict__ w, const float *__restrict__ x, float *__restrict__ y,
                                int K, int M, int64_t R, int64_t N, int64_t wbs, int plain, int flavor) {
  int64_t total = R * (int64_t)M;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += stride) {
    int64_t r = t / M;
    int m = (int)(t % M);
    const float *wr = w + (r / N) * wbs + (int64_t)m * K;
    const float *xr = x + r * K;
    if (plain) {
      float s = 0.0f;
      for (int i = 0; i < K; i++) s = __fadd_rn(s, __fmul_rn(wr[i], xr[i]));
      y[t] = arm_nan(s);
      continue;
    }
    float a[16];
#pragma unroll
    for (int j = 0; j < 16; j++) a[j] = 0.0f;
    int np = K & ~15;
    for (int i = 0; i < np; i += 16) {
#pragma unroll
      for (int j = 0; j < 16; j++) a[j] = __fmaf_rn(wr[i + j], xr[i + j], a[j]);
    }
#pragma unroll
    for (int l = 0; l < 4; l++) a[l] = __fadd_rn(a[l], a[8 + l]);
#pragma unroll
    for (int l = 0; l < 4; l++) a[4 + l] = __fadd_rn(a[4 + l], a[12 + l]);
#pragma unroll
    for (int l = 0; l < 4; l++) a[l] = __fadd_rn(a[l], a[4 + l]);
    float sumf = __fadd_rn(__fadd_rn(a[0], a[1]), __fadd_rn(a[2], a[3]));
    y[t] = arm_nan(dot_tail(wr, xr, np, K, sumf, flavor));
  }
}

// Pack `rows` rows of K floats (per batch) into dst[batch][Kq][rows_p], K reordered
// class-major (leaf order) over the first np = 16*seg elements, each segment
// padded to segp with `pad`; rows in [rows, rows_p) hold 0 (pad in the padding
// chunks). rows_p is a multiple of 64.
//
// One warp packs one 16-k chunk c of 64 rows. Lane (q = lane & 3, g = lane >> 2)
// loads, for each of two 32-row groups, rows 4g..4g+3 at k = 16c + 4q .. 16c + 4q + 3
// (16-byte loads when VEC), transposes the 4x4 block in registers and stores, for
// each of its classes j = 4q + e, the four rows as one 16-byte vector at packed
// row leaf(j)*segp + c: the 8 lanes of one q write 128 contiguous bytes. No
// shared memory; 8 loads per lane are in flight before the first store.
// Grid: (rows_p / 64, ceil(segp / 8), batches), 256 threads.
template <bool VEC>
__global__ void __launch_bounds__(256) k_mm_pack(const float *__restrict__ src, int rows, int K, int64_t src_batch,
                                                 int seg, int segp, int rows_p, float pad, float *__restrict__ dst) {
  const int lane = threadIdx.x & 31, q = lane & 3, g = lane >> 2;
  const int c = blockIdx.y * 8 + (threadIdx.x >> 5);
  if (c >= segp) return;
  const float *s = src + (int64_t)blockIdx.z * src_batch;
  float *d = dst + (int64_t)blockIdx.z * (16 * (int64_t)segp) * rows_p;
  float v[2][4][4];  // [group][row i][class e]
#pragma unroll
  for (int h = 0; h < 2; h++) {
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int r = blockIdx.x * 64 + 32 * h + 4 * g + i;
      if (c < seg && r < rows) {
        const float *p = s + (int64_t)r * K + 16 * c + 4 * q;
        if (VEC) {
          const float4 t = __ldg(reinterpret_cast<const float4 *>(p));
          v[h][i][0] = t.x; v[h][i][1] = t.y; v[h][i][2] = t.z; v[h][i][3] = t.w;
        } else {
#pragma unroll
          for (int e = 0; e < 4; e++) v[h][i][e] = __ldg(p + e);
        }
      } else {
#pragma unroll
        for (int e = 0; e < 4; e++) v[h][i][e] = c < seg ? 0.0f : pad;
      }
    }
  }
#pragma unroll
  for (int h = 0; h < 2; h++) {
    const int r = blockIdx.x * 64 + 32 * h + 4 * g;
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const int kq = leaf_of_class(4 * q + e) * segp + c;
      *reinterpret_cast<float4 *>(d + (int64_t)kq * rows_p + r) =
          make_float4(v[h][0][e], v[h][1][e], v[h][2][e], v[h][3][e]);
    }
  }
}

// Launch the pack of `batches` operands of `rows` x K (batch stride src_batch).
static cudaError_t launch_pack(const float *src, int rows, int K, int64_t src_batch, int batches, int seg, int segp,
                               int rows_p, float pad, float *dst, cudaStream_t stream) {
  dim3 grid(rows_p / 64, (segp + 7) / 8, batches);
  const bool vec = K % 4 == 0 && src_batch % 4 == 0 && ((uintptr_t)src & 15) == 0;
  if (vec)
    k_mm_pack<true><<<grid, 256, 0, stream>>>(src, rows, K, src_batch, seg, segp, rows_p, pad, dst);
  else
    k_mm_pack<false><<<grid, 256, 0, stream>>>(src, rows, K, src_batch, seg, segp, rows_p, pad, dst);
  return cudaGetLastError();
}

namespace mm {
constexpr int BM = 128;  // w rows (m) per CTA
constexpr int BN = 64;   // x rows (r) per CTA
constexpr int BK = 16;   // packed k per stage
constexpr int NS = 4;    // pipeline stages
constexpr int THREADS = 256;
constexpr int TM = 4, TN = 8;
constexpr int STAGE_FLOATS = BK * (BM + BN);
}  // namespace mm

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
  uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// Fold the finished chain of leaf S into the stack (post-order of the tree).
template <int S>
__device__ __forceinline__ void fold(float (&run)[mm::TM * mm::TN], float (&st)[4][mm::TM * mm::TN]) {
  constexpr int L0 = (S & 1) ? 1 : 0;
  constexpr int L1 = (S & 3) == 3 ? 1 : 0;
  constexpr int L2 = (S & 7) == 7 ? 1 : 0;
  constexpr int L3 = (S & 15) == 15 ? 1 : 0;
#pragma unroll
  for (int i = 0; i < mm::TM * mm::TN; i++) {
    float v = run[i];
    if (!L0) { st[0][i] = v; continue; }
    v = __fadd_rn(st[0][i], v);
    if (!L1) { st[1][i] = v; continue; }
    v = __fadd_rn(st[1][i], v);
    if (!L2) { st[2][i] = v; continue; }
    v = __fadd_rn(st[2][i], v);
    if (!L3) { st[3][i] = v; continue; }
    run[i] = __fadd_rn(st[3][i], v);  // the whole tree: sumf
  }
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
  int *ctr;           // k_mul_mat_tm in quarters: arrivals per tile (0 between launches)
};

enum { EP_BIAS = 1, EP_BIAS_LHS = 2, EP_RES = 4, EP_RES_LHS = 8 };

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

// The same adds over a finished y of R x M (the paths without a fused epilogue).
__global__ void k_mm_epilogue(MMArgs a, int64_t R) {
  const int64_t n = R * a.M;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    a.y[i] = epilogue_adds(a, a.y[i], i / a.M, (int)(i % a.M));
}

__global__ void __launch_bounds__(mm::THREADS, 1) k_mul_mat_fast(MMArgs a) {
  using namespace mm;
  extern __shared__ __align__(16) float smem[];
  const int tid = threadIdx.x;
  // Warps tile the CTA 4 (m) x 2 (r); lanes tile a warp 8 (m) x 4 (r), so a
  // warp's operand reads per k-step are one 128-byte w row and two 128-byte x
  // rows (broadcast within the lane groups).
  const int warp = tid >> 5, lane = tid & 31;
  const int tm = (warp & 3) * 8 + (lane & 7);   // m group: m = m0 + 4*tm + [0,4)
  const int tn = (warp >> 2) * 4 + (lane >> 3); // r group: r = r0 + 8*tn + [0,8)
  const int m0 = blockIdx.x * BM;
  const int bx = blockIdx.y / a.r_tiles;          // batch
  const int rt = blockIdx.y % a.r_tiles;
  const int64_t rl0 = (int64_t)rt * BN;            // first row within the batch
  const int Kq = 16 * a.segp;
  const float *wp = a.wp + (a.wbs ? (int64_t)bx * Kq * a.Mp : 0) + m0;
  const float *xp = a.xp + (int64_t)bx * Kq * a.Np + rl0;
  const int nstages = Kq / BK;

  auto issue = [&](int st) {
    float *ws = smem + (st % NS) * STAGE_FLOATS;
    float *xs = ws + BK * BM;
    const int k0 = st * BK;
    // 16 x 128 floats of w and 16 x 64 of x: 768 16-byte copies, three per thread.
#pragma unroll
    for (int i = 0; i < 3; i++) {
      int q = tid + i * THREADS;
      if (q < BK * BM / 4) {
        int row = q / (BM / 4), col = (q % (BM / 4)) * 4;
        cp_async16(ws + row * BM + col, wp + (int64_t)(k0 + row) * a.Mp + col);
      } else {
        q -= BK * BM / 4;
        int row = q / (BN / 4), col = (q % (BN / 4)) * 4;
        cp_async16(xs + row * BN + col, xp + (int64_t)(k0 + row) * a.Np + col);
      }
    }
  };

#pragma unroll
  for (int s = 0; s < NS - 1; s++) {
    if (s < nstages) issue(s);
    cp_async_commit();
  }

  float run[TM * TN];
  float st[4][TM * TN];
  const int groups_per_seg = a.segp / 4;
  int g = 0;  // global group (4 packed k-steps) index

#pragma unroll
  for (int S = 0; S < 16; S++) {
#pragma unroll
    for (int i = 0; i < TM * TN; i++) run[i] = 0.0f;
    for (int gi = 0; gi < groups_per_seg; gi++, g++) {
      const int stg = g >> 2;
      if ((g & 3) == 0) {
        cp_async_wait<NS - 2>();
        __syncthreads();
        if (stg + NS - 1 < nstages) issue(stg + NS - 1);
        cp_async_commit();
      }
      const float *ws = smem + (stg % NS) * STAGE_FLOATS;
      const float *xs = ws + BK * BM;
      const int row0 = (g & 3) * 4;
#pragma unroll
      for (int kk = 0; kk < 4; kk++) {
        const float4 wv = *reinterpret_cast<const float4 *>(ws + (row0 + kk) * BM + tm * 4);
        const float4 x0 = *reinterpret_cast<const float4 *>(xs + (row0 + kk) * BN + tn * 8);
        const float4 x1 = *reinterpret_cast<const float4 *>(xs + (row0 + kk) * BN + tn * 8 + 4);
        const float wr[4] = {wv.x, wv.y, wv.z, wv.w};
        const float xr[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
        for (int j = 0; j < TN; j++)
#pragma unroll
          for (int i = 0; i < TM; i++) run[j * TM + i] = __fmaf_rn(wr[i], xr[j], run[j * TM + i]);
      }
    }
    switch (S) {
      case 0: fold<0>(run, st); break;
      case 1: fold<1>(run, st); break;
      case 2: fold<2>(run, st); break;
      case 3: fold<3>(run, st); break;
      case 4: fold<4>(run, st); break;
      case 5: fold<5>(run, st); break;
      case 6: fold<6>(run, st); break;
      case 7: fold<7>(run, st); break;
      case 8: fold<8>(run, st); break;
      case 9: fold<9>(run, st); break;
      case 10: fold<10>(run, st); break;
      case 11: fold<11>(run, st); break;
      case 12: fold<12>(run, st); break;
      case 13: fold<13>(run, st); break;
      case 14: fold<14>(run, st); break;
      default: fold<15>(run, st); break;
    }
  }
  cp_async_wait<0>();

  // Epilogue: the tail (K mod 16 elements, in order) and the store.
  const int64_t rbase = (int64_t)bx * a.Nx;
#pragma unroll
  for (int j = 0; j < TN; j++) {
    const int64_t rl = rl0 + tn * 8 + j;
    if (rl >= a.Nx) continue;
    const int64_t r = rbase + rl;
#pragma unroll
    for (int i = 0; i < TM; i++) {
      const int m = m0 + tm * 4 + i;
      if (m >= a.M) continue;
      float v = run[j * TM + i];
      if (a.np < a.K) {
        const float *wr = a.w + (a.wbs ? (int64_t)bx * a.wbs : 0) + (int64_t)m * a.K;
        const float *xr = a.x + r * a.K;
        v = dot_tail(wr, xr, a.np, a.K, v, a.flavor);
      }
      a.y[r * a.M + m] = arm_nan(v);
    }
  }
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
  static constexpr size_t SMEM = (size_t)NS * Tile<WM>::STAGE_FLOATS * 4 + (size_t)LEVEL_FLOATS * 4;
  // A CTA that computes a quarter of the tree needs no level-2 slab: the same
  // shared memory holds more stages.
  static constexpr int NS_QUARTER = (int)(SMEM / (Tile<WM>::STAGE_FLOATS * 4));
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

// Fold the finished chain of leaf S into the stack: pop and add the levels
// below the first zero bit of S (the left operand is the older value, as in the
// tree), then push at that level. Levels 0 and 1 are TMEM columns tcol + 64 L;
// level 2 is this thread's float4 slots of the shared-memory slab lv2, float4 j
// of chunk c at lv2[(c * 4 + j) * THREADS] (consecutive threads, consecutive
// float4: no bank conflicts). Level 3 is pushed only at S = 7 (depth 3) and
// popped only at S = 15 (depth 4); the caller parks it in global memory, so
// here depth 3 leaves the value in acc and depth 4 stops after level 2.
__device__ __forceinline__ void tfold_rt(float2 (&acc2)[32], uint32_t tcol, float4 *lv2, int S, bool last = false) {
  const int depth = last ? 2 : __ffs(~S) - 1;  // trailing one bits: 0..4 (a quarter's last: pop 0 and 1)
  const int pops = depth < 3 ? depth : 3;
#pragma unroll
  for (int c = 0; c < 4; c++) {
    float v[16];
#pragma unroll
    for (int q = 0; q < 8; q++) {
      v[2 * q] = acc2[8 * c + q].x;
      v[2 * q + 1] = acc2[8 * c + q].y;
    }
    for (int L = 0; L < pops; L++) {
      float t[16];
      if (L < 2) {
        tmem_ld16(tcol + 64 * L + 16 * c, t);
      } else {
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const float4 u = lv2[(c * 4 + j) * mt::THREADS];
          t[4 * j] = u.x; t[4 * j + 1] = u.y; t[4 * j + 2] = u.z; t[4 * j + 3] = u.w;
        }
      }
#pragma unroll
      for (int i = 0; i < 16; i++) v[i] = __fadd_rn(t[i], v[i]);
    }
    if (depth < 2) {
      tmem_st16(tcol + 64 * depth + 16 * c, v);
    } else if (depth == 2 && !last) {
#pragma unroll
      for (int j = 0; j < 4; j++) lv2[(c * 4 + j) * mt::THREADS] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    }
#pragma unroll
    for (int q = 0; q < 8; q++) acc2[8 * c + q] = make_float2(v[2 * q], v[2 * q + 1]);
  }
}

// One CTA per tile, m-tile fastest (the CTAs running together share their x
// tile in L2).
// STAGE_FOLD: every segment spans whole stages (segp a multiple of 16), so the
// fold check runs once per stage; otherwise after every group of 4 k.
// QUARTER: the grid has four CTAs a tile, CTA q computing the subtree
// T(4q..4q+3) of segments 4q..4q+3 (a 2-level stack, all in TMEM); each writes
// its partial to a per-tile slice of a.park, and the last of the four to
// arrive (an atomic count, no waiting) adds ((T0 + T1) + (T2 + T3)) -- the top
// two levels of ggml's tree -- and runs the epilogue. Four times the CTAs fill
// the last wave of a grid that would leave SMs idle.
// EPI: the fused bias / residual adds in the epilogue (a separate instance, so
// the plain product compiles without them).
template <int WM, bool STAGE_FOLD, bool QUARTER, bool EPI>
__global__ void __launch_bounds__(mt::THREADS, mt::CTAS_PER_SM) k_mul_mat_tm(MMArgs a) {
  using namespace mt;
  constexpr int BM = Tile<WM>::BM, BN = Tile<WM>::BN, STAGE_FLOATS = Tile<WM>::STAGE_FLOATS;
  constexpr int NS = QUARTER ? Pipe<WM>::NS_QUARTER : Pipe<WM>::NS;
  extern __shared__ __align__(16) float smem[];
  __shared__ uint32_t tmem_base;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Warps WM (m) x 8/WM (r), lanes 8 (m) x 4 (r); a thread's m are mo + [0,4)
  // and mo + 32 + [0,4), its r are ro + [0,4) and ro + 16 + [0,4).
  const int mo = (warp % WM) * 64 + (lane & 7) * 4;
  const int ro = (warp / WM) * 32 + (lane >> 3) * 4;
  // This CTA's tile: m0, batch bx, first row rl0 (recomputed where needed, so
  // nothing but the operand pointers stays live through the k-loop).
  auto pos = [&](int &m0, int &bx, int64_t &rl0) {
    const int mtiles = a.Mp / BM, tile = QUARTER ? blockIdx.x >> 2 : blockIdx.x;
    m0 = (tile % mtiles) * BM;
    bx = (tile / mtiles) / a.r_tiles;
    rl0 = (int64_t)((tile / mtiles) % a.r_tiles) * BN;
  };
  const int Kq = 16 * a.segp;
  // A quarter reads packed k rows [4 q segp, 4 (q + 1) segp): its four segments.
  const int kq0 = QUARTER ? (int)(blockIdx.x & 3) * 4 * a.segp : 0;
  const float *wp, *xp;
  {
    int m0, bx;
    int64_t rl0;
    pos(m0, bx, rl0);
    wp = a.wp + (a.wbs ? (int64_t)bx * Kq * a.Mp : 0) + (int64_t)kq0 * a.Mp + m0;
    xp = a.xp + (int64_t)bx * Kq * a.Np + (int64_t)kq0 * a.Np + rl0;
  }
  const int nstages = (QUARTER ? Kq / 4 : Kq) / BK;

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

  // Stage copies: this thread moves w rows tid / (BM/4) + j (1024/BM), x rows
  // tid / (BN/4) + j (1024/BN), 16 bytes at column 4 (tid % (BM/4 or BN/4)).
  // The addresses are rebuilt at every stage (once per 16 k) rather than kept
  // live through the k-loop.
  constexpr int WCP = BM / 64, XCP = BN / 64;  // 16-byte copies a thread a stage
  auto issue = [&](int st) {
    const int t = threadIdx.x;
    float *sb = smem + (st % NS) * STAGE_FLOATS;
    const int64_t k0 = (int64_t)st * BK;
    const float *gw = wp + (k0 + t / (BM / 4)) * a.Mp + (t % (BM / 4)) * 4;
    const float *gx = xp + (k0 + t / (BN / 4)) * a.Np + (t % (BN / 4)) * 4;
    float *dw = sb + (t / (BM / 4)) * BM + (t % (BM / 4)) * 4;
    float *dx = sb + BK * BM + (t / (BN / 4)) * BN + (t % (BN / 4)) * 4;
#pragma unroll
    for (int j = 0; j < WCP; j++) cp_async16(dw + j * (1024 / BM) * BM, gw + (int64_t)j * (1024 / BM) * a.Mp);
#pragma unroll
    for (int j = 0; j < XCP; j++) cp_async16(dx + j * (1024 / BN) * BN, gx + (int64_t)j * (1024 / BN) * a.Np);
  };

#pragma unroll
  for (int s = 0; s < NS - 1; s++) {
    if (s < nstages) issue(s);
    cp_async_commit();
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
        p0 = make_float2(__fadd_rn(l3.x, p0.x), __fadd_rn(l3.y, p0.y));
        p1 = make_float2(__fadd_rn(l3.z, p1.x), __fadd_rn(l3.w, p1.y));
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
  auto end_group = [&]() {
    if (--gleft == 0) {
      tfold_rt(acc2, tcol, lv2, S, QUARTER && S == 3);
      gleft = a.segp / 4;
      // After S = 7 the fold left T(0..7) in acc (depth 3 pushes nothing).
      if (!QUARTER && S == 7) park(false);
      if (++S < (QUARTER ? 4 : 16)) {
#pragma unroll
        for (int i = 0; i < 32; i++) acc2[i] = make_float2(0.0f, 0.0f);
      }
    }
  };
  int so = 0;  // offset of stage st % NS
  for (int st = 0; st < nstages; st++) {
    cp_async_wait<NS - 2>();
    __syncthreads();
    if (st + NS - 1 < nstages) issue(st + NS - 1);
    cp_async_commit();
    const float *ws = smem + so + mo;
    const float *xs = smem + so + BK * BM + ro;
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
      if (!STAGE_FOLD) end_group();
    }
    if (STAGE_FOLD) {
      gleft -= GPS - 1;
      end_group();
    }
    so = so + STAGE_FLOATS == NS * STAGE_FLOATS ? 0 : so + STAGE_FLOATS;
  }
  cp_async_wait<0>();

  // Every TMEM access of this CTA is complete (each waited): free the columns.
  asm volatile("tcgen05.fence::before_thread_sync;\n");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;\n");
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem_base), "n"(TMEM_COLS));

  if (QUARTER) {
    // This quarter's T(4q..4q+3) to its slice; the last of the tile's four adds
    // the top of the tree.
    __shared__ int last;
    const int tile = blockIdx.x >> 2, q = blockIdx.x & 3;
    float4 *mine = reinterpret_cast<float4 *>(a.park + (size_t)blockIdx.x * (THREADS * 64)) + tid;
#pragma unroll
    for (int i = 0; i < 16; i++) mine[i * THREADS] = make_float4(acc2[2 * i].x, acc2[2 * i].y, acc2[2 * i + 1].x, acc2[2 * i + 1].y);
    __threadfence();
    __syncthreads();
    if (tid == 0) last = atomicAdd(a.ctr + tile, 1) == 3;
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (tid == 0) a.ctr[tile] = 0;  // ready for the next launch
    const float4 *base = reinterpret_cast<const float4 *>(a.park + (size_t)tile * 4 * (THREADS * 64)) + tid;
    (void)q;
#pragma unroll
    for (int i = 0; i < 16; i++) {
      // all four partials from L2 (this CTA's own too: it wrote them above)
      const float4 p0 = __ldcg(base + i * THREADS), p1 = __ldcg(base + 16 * THREADS + i * THREADS);
      const float4 p2 = __ldcg(base + 32 * THREADS + i * THREADS), p3 = __ldcg(base + 48 * THREADS + i * THREADS);
      auto add4 = [](float4 u, float4 v) {
        return make_float4(__fadd_rn(u.x, v.x), __fadd_rn(u.y, v.y), __fadd_rn(u.z, v.z), __fadd_rn(u.w, v.w));
      };
      const float4 r = add4(add4(p0, p1), add4(p2, p3));
      acc2[2 * i] = make_float2(r.x, r.y);
      acc2[2 * i + 1] = make_float2(r.z, r.w);
    }
  } else {
    // The root of the tree: T(0..7) + T(8..15).
    park(true);
  }
  // Epilogue: the tail (K mod 16 elements, in order) and the store.
  int m0, bx;
  int64_t rl0;
  pos(m0, bx, rl0);
  const int64_t rbase = (int64_t)bx * a.Nx;
  const bool vec = (a.M & 3) == 0;
  if constexpr (EPI) {
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
    for (int i = 0; i < 8; i++) acc[i] = make_float2(__fadd_rn(st[L][i].x, acc[i].x), __fadd_rn(st[L][i].y, acc[i].y));
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

// $SHLO_MUL_MAT_PATH = naive | fast forces one of the two exact paths (both give
// the same bits; the tests run each); unset, the size decides.
static int mm_path() {
  const char *e = getenv("SHLO_MUL_MAT_PATH");
  if (e && !strcmp(e, "naive")) return 1;
  if (e && !strcmp(e, "fast")) return 2;
  return 0;
}

static int pack_operand(Device *dev, const float *src, int rows, int K, int64_t src_batch, int batches, int seg,
                        int segp, int rows_p, float pad, Buffer **out) {
  size_t bytes = (size_t)batches * 16 * segp * rows_p * sizeof(float);
  SHLO_TRY(buffer_alloc(dev, bytes, out));
  launch_pack(src, rows, K, src_batch, batches, seg, segp, rows_p, pad, (float *)(*out)->ptr, dev->stream);
  if (launch_check("mul_mat pack")) {
    buffer_release(*out);
    return 1;
  }
  return 0;
}

int k_mul_mat(Device *dev, Arr *w, Arr *x, const uint32_t *p, Arr **out) {
  return k_mul_mat_ep(dev, w, x, p, nullptr, nullptr, 0, out);
}

int k_mul_mat_ep(Device *dev, Arr *w, Arr *x, const uint32_t *p, Arr *bias, Arr *res, int ep, Arr **out) {
  const int64_t K = p[0], M = p[1], R = p[2], wbs = p[3], N = p[4];
  const int plain = p[5] != 0;
  if ((ep & EP_BIAS) && (!bias || require_dtype(bias, kF32, "mul_mat bias") || check_elems(bias, M, "mul_mat bias")))
    return 1;
  if ((ep & EP_RES) && (!res || require_dtype(res, kF32, "mul_mat residual") || check_elems(res, R * M, "mul_mat residual")))
    return 1;
  MMArgs ea{};
  ea.bias = (ep & EP_BIAS) ? (const float *)data_ptr(bias) : nullptr;
  ea.res = (ep & EP_RES) ? (const float *)data_ptr(res) : nullptr;
  ea.ep = ep;
  SHLO_TRY(require_dtype(w, kF32, "mul_mat") || require_dtype(x, kF32, "mul_mat"));
  if (K <= 0 || N <= 0 || R % N) return fail("mul_mat: K=%lld R=%lld N=%lld not carried", (long long)K, (long long)R, (long long)N);
  const int64_t nb = R / N;
  SHLO_TRY(check_elems(x, R * K, "mul_mat x"));
  SHLO_TRY(check_elems(w, (wbs ? (nb - 1) * wbs : 0) + M * K, "mul_mat w"));
  if (wbs && wbs < M * K) return fail("mul_mat: w batch stride %lld below M*K", (long long)wbs);
  int64_t shape[1] = {R * M};
  Arr *o;
  SHLO_TRY(new_array(dev, kF32, shape, 1, &o));
  const int flavor = current_flavor();
  const int64_t np = K & ~(int64_t)15;
  int path = mm_path();
  bool fast = !plain && np >= 16 && (path == 2 || (path == 0 && R * M >= 4096));
  if (R * M == 0) {
    *out = o;
    return 0;
  }
  if (!fast) {
    k_mul_mat_naive<<<grid_for(R * M, 256, dev), 256, 0, dev->stream>>>(
        (const float *)data_ptr(w), (const float *)data_ptr(x), (float *)o->buf->ptr, (int)K, (int)M, R, N, wbs, plain,
        flavor);
    int rc = launch_check("mul_mat");
    if (!rc && ep) {
      ea.y = (float *)o->buf->ptr;
      ea.M = (int)M;
      k_mm_epilogue<<<grid_for(R * M, 256, dev), 256, 0, dev->stream>>>(ea, R);
      rc = launch_check("mul_mat epilogue");
    }
    if (rc) {
      shlo_release(o);
      return 1;
    }
    *out = o;
    return 0;
  }
  const int seg = (int)(np / 16);
  const int segp = (seg + 3) & ~3;
  // k_mul_mat_short (register stack, 64 x 64 tiles): every segment 4 packed k,
  // or up to 16 when M <= 64 (attention's value product).
  const bool short_k = segp == 4 || (M <= 64 && segp <= 16);
  const int WM = M <= 64 ? 1 : 2;
  const int BM = short_k ? ms::BM : WM == 1 ? mt::Tile<1>::BM : mt::Tile<2>::BM;
  const int BN = short_k ? ms::BN : WM == 1 ? mt::Tile<1>::BN : mt::Tile<2>::BN;
  const int Mp = (int)((M + BM - 1) / BM * BM);
  const int64_t Bx = wbs ? nb : 1;
  const int64_t Nx = wbs ? N : R;
  const int Np = (int)((Nx + BN - 1) / BN * BN);
  const int Wb = wbs ? (int)nb : 1;
  // The packed w is derived from w's storage, which never changes: keep it.
  Buffer *wpk = nullptr;
  {
    char key[160];
    snprintf(key, sizeof key, "mm:%lld:%lld:%lld:%d:%lld:%d", (long long)w->offset, (long long)K, (long long)M, Wb,
             (long long)wbs, Mp);
    std::lock_guard<std::mutex> lk(w->buf->derived_mu);
    auto it = w->buf->derived.find(key);
    if (it != w->buf->derived.end()) {
      wpk = it->second;
      buffer_retain(wpk);
    } else {
      if (pack_operand(dev, (const float *)data_ptr(w), (int)M, (int)K, wbs, Wb, seg, segp, Mp, -0.0f, &wpk)) {
        shlo_release(o);
        return 1;
      }
      // Not while a capture records (the pack is then a node of the graph), nor
      // on a buffer a graph owns (it is rewritten by every replay).
      if (!w->buf->graph_owner && !dev->capturing) {
        buffer_retain(wpk);
        w->buf->derived[key] = wpk;
        const float *src = (const float *)data_ptr(w);
        float *dst = (float *)wpk->ptr;
        const int m = (int)M, k = (int)K;
        w->buf->rederive[key] = [=]() {
          launch_pack(src, m, k, wbs, Wb, seg, segp, Mp, -0.0f, dst, dev->stream);
          return launch_check("mul_mat pack");
        };
      }
    }
  }
  Buffer *xpk;
  if (pack_operand(dev, (const float *)data_ptr(x), (int)Nx, (int)K, Nx * K, (int)Bx, seg, segp, Np, 0.0f, &xpk)) {
    buffer_release(wpk);
    shlo_release(o);
    return 1;
  }
  MMArgs a = ea;
  a.wp = (const float *)wpk->ptr;
  a.xp = (const float *)xpk->ptr;
  a.w = (const float *)data_ptr(w);
  a.x = (const float *)data_ptr(x);
  a.y = (float *)o->buf->ptr;
  a.K = (int)K;
  a.M = (int)M;
  a.np = (int)np;
  a.segp = segp;
  a.Mp = Mp;
  a.Np = Np;
  a.Nx = Nx;
  a.wbs = wbs;
  a.r_tiles = Np / BN;
  a.flavor = flavor;
  a.bx_count = (int)Bx;
  if (short_k) {
    const unsigned grid = (unsigned)((int64_t)(Mp / BM) * Bx * a.r_tiles);
#define SHLO_MS(NG)                                                                  \
  (ep ? k_mul_mat_short<true, NG><<<grid, ms::THREADS, 0, dev->stream>>>(a)          \
      : k_mul_mat_short<false, NG><<<grid, ms::THREADS, 0, dev->stream>>>(a))
    switch (segp / 4) {
      case 1: SHLO_MS(1); break;
      case 2: SHLO_MS(2); break;
      case 3: SHLO_MS(3); break;
      default: SHLO_MS(4); break;
    }
#undef SHLO_MS
    int rc = launch_check("mul_mat");
    buffer_release(wpk);
    buffer_release(xpk);
    if (rc) {
      shlo_release(o);
      return 1;
    }
    *out = o;
    return 0;
  }
  const size_t smem = WM == 1 ? mt::Pipe<1>::SMEM : mt::Pipe<2>::SMEM;
  static bool attr_done[64] = {false};
  if (!attr_done[dev->id]) {
    int rc = 0;
    auto attr = [&](auto kern, size_t bytes) {
      if (!rc) rc = cuda_check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes),
                               "mul_mat attribute");
    };
    attr(k_mul_mat_tm<1, false, false, false>, mt::Pipe<1>::SMEM);
    attr(k_mul_mat_tm<1, true, false, false>, mt::Pipe<1>::SMEM);
    attr(k_mul_mat_tm<2, false, false, false>, mt::Pipe<2>::SMEM);
    attr(k_mul_mat_tm<2, true, false, false>, mt::Pipe<2>::SMEM);
    attr(k_mul_mat_tm<1, false, true, false>, mt::Pipe<1>::SMEM);
    attr(k_mul_mat_tm<1, true, true, false>, mt::Pipe<1>::SMEM);
    attr(k_mul_mat_tm<2, false, true, false>, mt::Pipe<2>::SMEM);
    attr(k_mul_mat_tm<2, true, true, false>, mt::Pipe<2>::SMEM);
    attr(k_mul_mat_tm<1, false, false, true>, mt::Pipe<1>::SMEM);
    attr(k_mul_mat_tm<1, true, false, true>, mt::Pipe<1>::SMEM);
    attr(k_mul_mat_tm<2, false, false, true>, mt::Pipe<2>::SMEM);
    attr(k_mul_mat_tm<2, true, false, true>, mt::Pipe<2>::SMEM);
    attr(k_mul_mat_tm<1, false, true, true>, mt::Pipe<1>::SMEM);
    attr(k_mul_mat_tm<1, true, true, true>, mt::Pipe<1>::SMEM);
    attr(k_mul_mat_tm<2, false, true, true>, mt::Pipe<2>::SMEM);
    attr(k_mul_mat_tm<2, true, true, true>, mt::Pipe<2>::SMEM);
    if (rc) {
      buffer_release(wpk);
      buffer_release(xpk);
      shlo_release(o);
      return 1;
    }
    attr_done[dev->id] = true;
  }
  // Quarters when they fill the last wave of two-CTA-per-SM slots markedly
  // better ($SHLO_MM_SPLIT = 1 | 4 forces one form; both give the same bits).
  const int64_t tiles = (int64_t)(Mp / BM) * Bx * a.r_tiles;
  const int64_t slots = (int64_t)mt::CTAS_PER_SM * dev->sm_count;
  auto wave_fill = [&](int64_t t) { return (double)t / (double)(((t + slots - 1) / slots) * slots); };
  // (A quarter must be long enough to pay for its own pipeline fill and the
  // partials: segp >= 64, i.e. K >= 1024, sixteen stages a quarter.)
  bool quarter = segp >= 64 && wave_fill(4 * tiles) > wave_fill(tiles) + 0.04;
  if (const char *e = getenv("SHLO_MM_SPLIT")) quarter = atoi(e) == 4;
  const unsigned grid = (unsigned)(quarter ? 4 * tiles : tiles);
  Buffer *park, *ctr = nullptr;
  if (buffer_alloc(dev, (size_t)grid * mt::THREADS * 64 * sizeof(float), &park) ||
      (quarter && buffer_alloc(dev, (size_t)tiles * sizeof(int), &ctr)) ||
      (quarter && cuda_check(cudaMemsetAsync(ctr->ptr, 0, (size_t)tiles * sizeof(int), dev->stream), "mul_mat counters"))) {
    buffer_release(park);
    buffer_release(ctr);
    buffer_release(wpk);
    buffer_release(xpk);
    shlo_release(o);
    return 1;
  }
  a.park = (float *)park->ptr;
  a.ctr = quarter ? (int *)ctr->ptr : nullptr;
  const bool stage_fold = segp % 16 == 0;
#define SHLO_TM(WMv, SF, Q)                                                      \
  (ep ? k_mul_mat_tm<WMv, SF, Q, true><<<grid, mt::THREADS, smem, dev->stream>>>(a) \
      : k_mul_mat_tm<WMv, SF, Q, false><<<grid, mt::THREADS, smem, dev->stream>>>(a))
  if (WM == 1) {
    if (stage_fold) quarter ? SHLO_TM(1, true, true) : SHLO_TM(1, true, false);
    else quarter ? SHLO_TM(1, false, true) : SHLO_TM(1, false, false);
  } else {
    if (stage_fold) quarter ? SHLO_TM(2, true, true) : SHLO_TM(2, true, false);
    else quarter ? SHLO_TM(2, false, true) : SHLO_TM(2, false, false);
  }
#undef SHLO_TM
  int rc = launch_check("mul_mat");
  buffer_release(park);
  buffer_release(ctr);
  buffer_release(wpk);
  buffer_release(xpk);
  if (rc) {
    shlo_release(o);
    return 1;
  }
  *out = o;
  return 0;
}

// ============================================================== soft_max ====
// Shaders.lean:100-123 / ggml_compute_forward_soft_max_f32 with
// ggml_vec_soft_max_f32 (vec.cpp): wv = x*scale; max; each four-lane group
// e_l = ggml_v_expf(wv_l - max), y = e, part = (e0+e1)+(e2+e3); the parts are
// added to a binary64 sum in group order; inv = (float)(1.0/sum); y *= inv.
//
// One warp per row. The max is an exact order-free reduction: for rows without
// NaN it is the largest value, and which of +0/-0 it is cannot change any
// output (wv - max is then +-0 or the same nonzero value, and ggml_v_expf(+-0)
// is 1). Rows with a NaN take the sequential scan of the spec. The binary64
// sum is the spec's serial chain, run by lane 0 over the parts in order.
// Rows whose length is not a multiple of 4 are refused by the caller.

template <int G>  // float4 groups per lane kept in registers (0 = stream through memory)
__global__ void g_soft_max(const float *__restrict__ x, float *__restrict__ y, int ncols, int64_t rows, float sc,
                           int float_sum) {
  extern __shared__ double parts_all[];
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  const int wpb = blockDim.x >> 5;
  const int ng = ncols / 4;
  double *parts = parts_all + wib * (G > 0 ? G * 32 : 256);
  for (int64_t row = (int64_t)blockIdx.x * wpb + wib; row < rows; row += (int64_t)gridDim.x * wpb) {
    const float4 *xr = reinterpret_cast<const float4 *>(x + row * ncols);
    float4 *yr = reinterpret_cast<float4 *>(y + row * ncols);
    float4 v[G > 0 ? G : 1];
    float mx = -INFINITY;
    bool nan = false;
    if (G > 0) {
#pragma unroll
      for (int i = 0; i < G; i++) {
        int gi = lane + 32 * i;
        if (gi < ng) {
          float4 t = xr[gi];
          t.x = __fmul_rn(t.x, sc); t.y = __fmul_rn(t.y, sc); t.z = __fmul_rn(t.z, sc); t.w = __fmul_rn(t.w, sc);
          v[i] = t;
          nan |= (t.x != t.x) | (t.y != t.y) | (t.z != t.z) | (t.w != t.w);
          mx = fmaxf(mx, fmaxf(fmaxf(t.x, t.y), fmaxf(t.z, t.w)));
        }
      }
    } else {
      for (int gi = lane; gi < ng; gi += 32) {
        float4 t = xr[gi];
        t.x = __fmul_rn(t.x, sc); t.y = __fmul_rn(t.y, sc); t.z = __fmul_rn(t.z, sc); t.w = __fmul_rn(t.w, sc);
        nan |= (t.x != t.x) | (t.y != t.y) | (t.z != t.z) | (t.w != t.w);
        mx = fmaxf(mx, fmaxf(fmaxf(t.x, t.y), fmaxf(t.z, t.w)));
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (__any_sync(0xffffffffu, nan)) {
      if (lane == 0) {
        float m = -INFINITY;
        for (int i = 0; i < ncols; i++) {
          float wv = __fmul_rn(x[row * ncols + i], sc);
          m = (m > wv) ? m : wv;
        }
        mx = m;
      }
      mx = __shfl_sync(0xffffffffu, mx, 0);
    }
    double sum = 0.0;
    float fs = 0.0f;
    // Chunks of 32*max(G,8) groups: parts into shared memory, lane 0 chains them.
    const int chunk = 32 * (G > 0 ? G : 8);
    for (int c0 = 0; c0 < ng; c0 += chunk) {
#pragma unroll
      for (int i = 0; i < (G > 0 ? G : 8); i++) {
        int gi = c0 + lane + 32 * i;
        if (gi < ng) {
          float4 t;
          if (G > 0) {
            t = v[i];
          } else {
            t = xr[gi];
            t.x = __fmul_rn(t.x, sc); t.y = __fmul_rn(t.y, sc); t.z = __fmul_rn(t.z, sc); t.w = __fmul_rn(t.w, sc);
          }
          float4 e;
          e.x = ggml_v_expf(__fsub_rn(t.x, mx));
          e.y = ggml_v_expf(__fsub_rn(t.y, mx));
          e.z = ggml_v_expf(__fsub_rn(t.z, mx));
          e.w = ggml_v_expf(__fsub_rn(t.w, mx));
          if (G > 0) v[i] = e;
          else yr[gi] = e;
          // widened here, by every lane, so lane 0's chain is adds alone
          parts[lane + 32 * i] = (double)__fadd_rn(__fadd_rn(e.x, e.y), __fadd_rn(e.z, e.w));
        }
      }
      __syncwarp();
      if (lane == 0) {
        int n = ng - c0 < chunk ? ng - c0 : chunk;
        if (float_sum) {
          for (int k = 0; k < n; k++) fs = __fadd_rn(fs, (float)parts[k]);
        } else {
          // eight parts loaded ahead of their serial adds
          int k = 0;
          for (; k + 8 <= n; k += 8) {
            double v[8];
#pragma unroll
            for (int i = 0; i < 8; i++) v[i] = parts[k + i];
#pragma unroll
            for (int i = 0; i < 8; i++) sum = __dadd_rn(sum, v[i]);
          }
          for (; k < n; k++) sum = __dadd_rn(sum, parts[k]);
        }
      }
      __syncwarp();
    }
    float inv;
    if (lane == 0) inv = float_sum ? __fdiv_rn(1.0f, fs) : __double2float_rn(__ddiv_rn(1.0, sum));
    inv = __shfl_sync(0xffffffffu, inv, 0);
    if (G > 0) {
#pragma unroll
      for (int i = 0; i < G; i++) {
        int gi = lane + 32 * i;
        if (gi < ng) {
          float4 e = v[i];
          e.x = arm_nan(__fmul_rn(e.x, inv)); e.y = arm_nan(__fmul_rn(e.y, inv));
          e.z = arm_nan(__fmul_rn(e.z, inv)); e.w = arm_nan(__fmul_rn(e.w, inv));
          yr[gi] = e;
        }
      }
    } else {
      for (int gi = lane; gi < ng; gi += 32) {
        float4 e = yr[gi];
        e.x = arm_nan(__fmul_rn(e.x, inv)); e.y = arm_nan(__fmul_rn(e.y, inv));
        e.z = arm_nan(__fmul_rn(e.z, inv)); e.w = arm_nan(__fmul_rn(e.w, inv));
        yr[gi] = e;
      }
    }
    __syncwarp();
  }
}

int k_soft_max(Device *dev, Arr *x, const uint32_t *p, Arr **out) {
  const int64_t ncols = p[0], rows = p[1];
  const float sc = bitsf_host(p[2]);
  const int float_sum = p[3] != 0;
  SHLO_TRY(require_dtype(x, kF32, "soft_max"));
  if (ncols % 4)
    return fail("soft_max: a row of %lld has a %lld-element tail that ggml-cpu sends through the platform expf, "
                "which is not carried", (long long)ncols, (long long)(ncols % 4));
  SHLO_TRY(check_elems(x, ncols * rows, "soft_max"));
  int64_t shape[1] = {ncols * rows};
  Arr *o;
  SHLO_TRY(new_array(dev, kF32, shape, 1, &o));
  if (ncols * rows > 0) {
    const int wpb = 4;
    int64_t blocks = (rows + wpb - 1) / wpb;
    if (blocks > (int64_t)dev->sm_count * 16) blocks = (int64_t)dev->sm_count * 16;
    const float *xp = (const float *)data_ptr(x);
    float *yp = (float *)o->buf->ptr;
    int ng = (int)(ncols / 4);
    if (ng <= 32 * 2)
      g_soft_max<2><<<(unsigned)blocks, wpb * 32, wpb * 64 * sizeof(double), dev->stream>>>(xp, yp, (int)ncols, rows, sc, float_sum);
    else if (ng <= 32 * 8)
      g_soft_max<8><<<(unsigned)blocks, wpb * 32, wpb * 256 * sizeof(double), dev->stream>>>(xp, yp, (int)ncols, rows, sc, float_sum);
    else
      g_soft_max<0><<<(unsigned)blocks, wpb * 32, wpb * 256 * sizeof(double), dev->stream>>>(xp, yp, (int)ncols, rows, sc, float_sum);
    if (launch_check("soft_max")) {
      shlo_release(o);
      return 1;
    }
  }
  *out = o;
  return 0;
}

// ================================================================== norm ====
// Shaders.lean:130-166 / ggml_compute_forward_norm_f32 without Accelerate:
// sum = binary64 sum of the row in order; mean = (float)sum / (float)N (a
// correctly rounded binary32 division); s2 = binary64 sum, in order, of the
// four-lane groups (d0^2+d1^2)+(d2^2+d3^2), d = x - mean, then of the tail
// elements' d^2; var = (float)(s2 / N); scale = 1.0f / sqrtf(var + eps); y =
// (x - mean) * scale.
//
// Each warp owns 32 rows; lane l runs row l's two serial binary64 chains. The
// rows stream through a 32x33 shared-memory tile in chunks of 32 columns, so
// every global access is a coalesced row segment.

__global__ void g_norm(const float *__restrict__ x, float *__restrict__ y, int ncols, int64_t rows, float eps,
                       int gpu_ops) {
  __shared__ float tiles[8][32][33];
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  float(*tile)[33] = tiles[wib];
  const int64_t nblk = (rows + 31) / 32;
  for (int64_t blk = (int64_t)blockIdx.x * 8 + wib; blk < nblk; blk += (int64_t)gridDim.x * 8) {
    const int64_t r0 = blk * 32;
    const int nr = rows - r0 < 32 ? (int)(rows - r0) : 32;
    auto load_tile = [&](int c0) {
#pragma unroll 8
      for (int rr = 0; rr < 32; rr++) {
        float v = 0.0f;
        if (rr < nr && c0 + lane < ncols) v = x[(r0 + rr) * ncols + c0 + lane];
        tile[rr][lane] = v;
      }
      __syncwarp();
    };
    const int nb = ncols & ~3;
    double sum = 0.0;
    float fsum = 0.0f;
    for (int c0 = 0; c0 < ncols; c0 += 32) {
      load_tile(c0);
      int n = ncols - c0 < 32 ? ncols - c0 : 32;
      for (int c = 0; c < n; c++) {
        float v = tile[lane][c];
        sum = __dadd_rn(sum, (double)v);
        fsum = __fadd_rn(fsum, v);
      }
      __syncwarp();
    }
    float mean = gpu_ops ? __fdividef(fsum, (float)ncols) : __fdiv_rn(__double2float_rn(sum), (float)ncols);
    double s2 = 0.0;
    float fs2 = 0.0f;
    for (int c0 = 0; c0 < ncols; c0 += 32) {
      load_tile(c0);
      int n = ncols - c0 < 32 ? ncols - c0 : 32;
      int c = 0;
      for (; c + 3 < n && c0 + c + 3 < nb; c += 4) {
        float d0 = __fsub_rn(tile[lane][c], mean), d1 = __fsub_rn(tile[lane][c + 1], mean);
        float d2 = __fsub_rn(tile[lane][c + 2], mean), d3 = __fsub_rn(tile[lane][c + 3], mean);
        float q = __fadd_rn(__fadd_rn(__fmul_rn(d0, d0), __fmul_rn(d1, d1)), __fadd_rn(__fmul_rn(d2, d2), __fmul_rn(d3, d3)));
        s2 = __dadd_rn(s2, (double)q);
        fs2 = __fadd_rn(fs2, __fmul_rn(d0, d0));
        fs2 = __fadd_rn(fs2, __fmul_rn(d1, d1));
        fs2 = __fadd_rn(fs2, __fmul_rn(d2, d2));
        fs2 = __fadd_rn(fs2, __fmul_rn(d3, d3));
      }
      for (; c < n; c++) {
        float d = __fsub_rn(tile[lane][c], mean);
        float q = __fmul_rn(d, d);
        s2 = __dadd_rn(s2, (double)q);
        fs2 = __fadd_rn(fs2, q);
      }
      __syncwarp();
    }
    float scl;
    if (gpu_ops) {
      scl = __fdividef(1.0f, sqrtf(__fadd_rn(__fdividef(fs2, (float)ncols), eps)));
    } else {
      float var = __double2float_rn(__ddiv_rn(s2, (double)ncols));
      scl = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
    }
    for (int c0 = 0; c0 < ncols; c0 += 32) {
#pragma unroll 8
      for (int rr = 0; rr < 32; rr++) {
        // every lane takes part in the shuffles; only the store is predicated
        float m = __shfl_sync(0xffffffffu, mean, rr);
        float s = __shfl_sync(0xffffffffu, scl, rr);
        if (rr < nr && c0 + lane < ncols) {
          int64_t i = (r0 + rr) * ncols + c0 + lane;
          y[i] = arm_nan(__fmul_rn(__fsub_rn(x[i], m), s));
        }
      }
    }
  }
}

// The same computation with a block's rows resident in shared memory (ncols <=
// 1024, ncols % 4 == 0): NORM_ROWS rows per block of NORM_THREADS threads. All
// threads load the rows with 16-byte loads (NORM_UNROLL in flight per thread),
// lanes 0..NORM_ROWS-1 of warp 0 run the rows' serial chains from shared memory
// (row pitch ncols + 1: conflict-free), and all threads write the output with
// 16-byte stores.
constexpr int NORM_ROWS = 16, NORM_THREADS = 128, NORM_UNROLL = 4;

__global__ void __launch_bounds__(NORM_THREADS) g_norm_rows(const float *__restrict__ x, float *__restrict__ y,
                                                            int ncols, int64_t rows, float eps,
                                                            const float *__restrict__ gamma,
                                                            const float *__restrict__ beta) {
  extern __shared__ float tile[];  // [NORM_ROWS][ncols + 1]
  __shared__ float ms[NORM_ROWS], ss[NORM_ROWS];
  const int tid = threadIdx.x;
  const int pitch = ncols + 1;
  const int64_t r0 = (int64_t)blockIdx.x * NORM_ROWS;
  const int nr = rows - r0 < NORM_ROWS ? (int)(rows - r0) : NORM_ROWS;
  const int cv = ncols / 4;  // float4 per row
  const int nv = nr * cv;
  const float4 *xb = reinterpret_cast<const float4 *>(x + r0 * ncols);
  for (int v0 = tid; v0 < nv; v0 += NORM_THREADS * NORM_UNROLL) {
    float4 t[NORM_UNROLL];
#pragma unroll
    for (int u = 0; u < NORM_UNROLL; u++) {
      const int v = v0 + u * NORM_THREADS;
      if (v < nv) t[u] = __ldg(xb + v);
    }
#pragma unroll
    for (int u = 0; u < NORM_UNROLL; u++) {
      const int v = v0 + u * NORM_THREADS;
      if (v < nv) {
        const int r = v / cv, c = 4 * (v - r * cv);
        float *d = tile + r * pitch + c;
        d[0] = t[u].x; d[1] = t[u].y; d[2] = t[u].z; d[3] = t[u].w;
      }
    }
  }
  __syncthreads();
  if (tid < nr) {
    // The chains run several steps at a time with their operands loaded and
    // widened first, so only the binary64 adds are serial.
    const float *row = tile + tid * pitch;
    double sum = 0.0;
    int c = 0;
    for (; c + 8 <= ncols; c += 8) {
      double v[8];
#pragma unroll
      for (int i = 0; i < 8; i++) v[i] = (double)row[c + i];
#pragma unroll
      for (int i = 0; i < 8; i++) sum = __dadd_rn(sum, v[i]);
    }
    for (; c < ncols; c++) sum = __dadd_rn(sum, (double)row[c]);
    const float mean = __fdiv_rn(__double2float_rn(sum), (float)ncols);
    auto group = [&](int g) {
      float d0 = __fsub_rn(row[g], mean), d1 = __fsub_rn(row[g + 1], mean);
      float d2 = __fsub_rn(row[g + 2], mean), d3 = __fsub_rn(row[g + 3], mean);
      return (double)__fadd_rn(__fadd_rn(__fmul_rn(d0, d0), __fmul_rn(d1, d1)),
                               __fadd_rn(__fmul_rn(d2, d2), __fmul_rn(d3, d3)));
    };
    double s2 = 0.0;
    c = 0;
    for (; c + 16 <= ncols; c += 16) {  // ncols % 4 == 0: no tail
      double q[4];
#pragma unroll
      for (int i = 0; i < 4; i++) q[i] = group(c + 4 * i);
#pragma unroll
      for (int i = 0; i < 4; i++) s2 = __dadd_rn(s2, q[i]);
    }
    for (; c < ncols; c += 4) s2 = __dadd_rn(s2, group(c));
    const float var = __double2float_rn(__ddiv_rn(s2, (double)ncols));
    ms[tid] = mean;
    ss[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
  }
  __syncthreads();
  float4 *yb = reinterpret_cast<float4 *>(y + r0 * ncols);
  for (int v = tid; v < nv; v += NORM_THREADS) {
    const int r = v / cv, c = 4 * (v - r * cv);
    const float *s = tile + r * pitch + c;
    const float m = ms[r], k = ss[r];
    float4 o;
    o.x = arm_nan(__fmul_rn(__fsub_rn(s[0], m), k));
    o.y = arm_nan(__fmul_rn(__fsub_rn(s[1], m), k));
    o.z = arm_nan(__fmul_rn(__fsub_rn(s[2], m), k));
    o.w = arm_nan(__fmul_rn(__fsub_rn(s[3], m), k));
    if (gamma) {  // the executor's fused affine: (y * gamma) + beta, each rounded alone
      const float4 g = __ldg(reinterpret_cast<const float4 *>(gamma + c));
      const float4 b = __ldg(reinterpret_cast<const float4 *>(beta + c));
      o = make_float4(__fadd_rn(__fmul_rn(o.x, g.x), b.x), __fadd_rn(__fmul_rn(o.y, g.y), b.y),
                      __fadd_rn(__fmul_rn(o.z, g.z), b.z), __fadd_rn(__fmul_rn(o.w, g.w), b.w));
    }
    yb[v] = o;
  }
}

// (y * gamma[c]) + beta[c] in place, for the norm path without a fused affine.
__global__ void k_affine_rows(float *y, int64_t n, int ncols, const float *gamma, const float *beta) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % ncols);
    y[i] = __fadd_rn(__fmul_rn(y[i], gamma[c]), beta[c]);
  }
}

int k_norm(Device *dev, Arr *x, const uint32_t *p, Arr **out) { return k_norm_affine(dev, x, p, nullptr, nullptr, out); }

int k_norm_affine(Device *dev, Arr *x, const uint32_t *p, Arr *gamma, Arr *beta, Arr **out) {
  const int64_t ncols = p[0], rows = p[1];
  const float eps = bitsf_host(p[2]);
  SHLO_TRY(require_dtype(x, kF32, "norm"));
  SHLO_TRY(check_elems(x, ncols * rows, "norm"));
  const bool affine = gamma != nullptr;
  if (affine) {
    SHLO_TRY(require_dtype(gamma, kF32, "norm gamma") || check_elems(gamma, ncols, "norm gamma"));
    SHLO_TRY(require_dtype(beta, kF32, "norm beta") || check_elems(beta, ncols, "norm beta"));
  }
  const float *gp = affine ? (const float *)data_ptr(gamma) : nullptr;
  const float *bp = affine ? (const float *)data_ptr(beta) : nullptr;
  int64_t shape[1] = {ncols * rows};
  Arr *o;
  SHLO_TRY(new_array(dev, kF32, shape, 1, &o));
  const size_t smem = (size_t)NORM_ROWS * (ncols + 1) * sizeof(float);
  const bool aligned = (((uintptr_t)data_ptr(x)) & 15) == 0 &&
                       (!affine || ((((uintptr_t)gp) | ((uintptr_t)bp)) & 15) == 0);
  if (ncols * rows > 0 && p[3] == 0 && ncols % 4 == 0 && ncols <= 1024 && aligned) {
    static bool attr_done[64] = {false};
    if (!attr_done[dev->id]) {
      if (cuda_check(cudaFuncSetAttribute(g_norm_rows, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          NORM_ROWS * 1025 * (int)sizeof(float)), "norm attribute")) {
        shlo_release(o);
        return 1;
      }
      attr_done[dev->id] = true;
    }
    g_norm_rows<<<(unsigned)((rows + NORM_ROWS - 1) / NORM_ROWS), NORM_THREADS, smem, dev->stream>>>(
        (const float *)data_ptr(x), (float *)o->buf->ptr, (int)ncols, rows, eps, gp, bp);
    if (launch_check("norm")) {
      shlo_release(o);
      return 1;
    }
  } else if (ncols * rows > 0) {
    int64_t nblk = (rows + 31) / 32;
    int64_t blocks = (nblk + 7) / 8;
    if (blocks > (int64_t)dev->sm_count * 8) blocks = (int64_t)dev->sm_count * 8;
    g_norm<<<(unsigned)blocks, 256, 0, dev->stream>>>((const float *)data_ptr(x), (float *)o->buf->ptr, (int)ncols,
                                                       rows, eps, p[3] != 0);
    int rc = launch_check("norm");
    if (!rc && affine) {
      k_affine_rows<<<grid_for(ncols * rows, 256, dev), 256, 0, dev->stream>>>((float *)o->buf->ptr, ncols * rows,
                                                                            (int)ncols, gp, bp);
      rc = launch_check("norm affine");
    }
    if (rc) {
      shlo_release(o);
      return 1;
    }
  }
  *out = o;
  return 0;
}

// =========================================================== elementwise ====

// Elementwise maps: each thread moves 16-byte vectors (two per trip for the
// one-input maps) in a grid-stride loop; the n mod 4 tail is done element by
// element. Every pointer is 16-byte aligned (fresh allocations, and kernel
// inputs are realigned by the API before the launch).
template <typename F>
__device__ __forceinline__ void map_f32(const float *__restrict__ x, float *__restrict__ y, int64_t n, F f) {
  const int64_t nv = n >> 2;
  const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, stride = (int64_t)gridDim.x * blockDim.x;
  const float4 *xv = reinterpret_cast<const float4 *>(x);
  float4 *yv = reinterpret_cast<float4 *>(y);
  int64_t i = t0;
  for (; i + stride < nv; i += 2 * stride) {
    const float4 a = __ldg(xv + i), b = __ldg(xv + i + stride);
    yv[i] = make_float4(f(a.x), f(a.y), f(a.z), f(a.w));
    yv[i + stride] = make_float4(f(b.x), f(b.y), f(b.z), f(b.w));
  }
  if (i < nv) {
    const float4 a = __ldg(xv + i);
    yv[i] = make_float4(f(a.x), f(a.y), f(a.z), f(a.w));
  }
  for (int64_t j = 4 * nv + t0; j < n; j += stride) y[j] = f(x[j]);
}

template <typename F>
__device__ __forceinline__ void map2_f32(const float *__restrict__ a, const float *__restrict__ b,
                                         float *__restrict__ y, int64_t n, F f) {
  const int64_t nv = n >> 2;
  const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = t0; i < nv; i += stride) {
    const float4 u = __ldg(reinterpret_cast<const float4 *>(a) + i), v = __ldg(reinterpret_cast<const float4 *>(b) + i);
    reinterpret_cast<float4 *>(y)[i] = make_float4(f(u.x, v.x), f(u.y, v.y), f(u.z, v.z), f(u.w, v.w));
  }
  for (int64_t j = 4 * nv + t0; j < n; j += stride) y[j] = f(a[j], b[j]);
}

// silu: Shaders.lean:172-179 (ggml_vec_silu_f32's four-lane body):
// y = x / (1 + ggml_v_expf(0 - x)), a correctly rounded division.
__device__ __forceinline__ float silu_one(float v, int gpu_ops) {
  if (gpu_ops) return __fdividef(v, __fadd_rn(1.0f, __expf(-v)));
  float r = __fdiv_rn(v, __fadd_rn(1.0f, ggml_v_expf(__fsub_rn(0.0f, v))));
  // arm64: a NaN input comes back quieted (every step passes it through); an
  // invalid division (-inf / inf) gives the default NaN.
  const uint32_t b = fbits(v);
  if ((b & 0x7FFFFFFFu) > 0x7F800000u) r = bitsf(b | 0x00400000u);
  else if (r != r) r = bitsf(0x7FC00000u);
  return r;
}

__global__ void g_silu(const float *__restrict__ x, float *__restrict__ y, int64_t n, int gpu_ops) {
  map_f32(x, y, n, [gpu_ops](float v) { return silu_one(v, gpu_ops); });
}

// gelu_erf: Shaders.lean:186-199 (ggml_vec_gelu_erf_f32):
// y = (0.5f*x) * (1.0f + erff(x*SQRT_2_INV)) with the correctly rounded erff; a
// NaN input returns itself quieted, as every arm64 step does.
__device__ __forceinline__ float gelu_one(float v, int gpu_erf, const shlo_erf::ErfSmem *t) {
  float ev;
  if (gpu_erf) {
    // The planted fault: GELU's tanh form (SQRT_2_OVER_PI, GELU_COEF_A of vec.h).
    ev = tanhf(__fmul_rn(__fmul_rn(bitsf(0x3F4C422Au), v),
                         __fadd_rn(1.0f, __fmul_rn(__fmul_rn(bitsf(0x3D372713u), v), v))));
  } else {
    ev = shlo_erf::erff_cr_smem(__fmul_rn(v, bitsf(0x3F3504F3u)), t);
  }
  float r = __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, ev));
  const uint32_t b = fbits(v);
  if ((b & 0x7FFFFFFFu) > 0x7F800000u) r = bitsf(b | 0x00400000u);
  else if (r != r) r = bitsf(0x7FC00000u);  // -inf * 0: arm64's default NaN
  return r;
}

__global__ void g_gelu_erf(const float *__restrict__ x, float *__restrict__ y, int64_t n, int gpu_erf) {
  __shared__ shlo_erf::ErfSmem tab;
  shlo_erf::erf_smem_load(&tab);
  __syncthreads();
  const shlo_erf::ErfSmem *t = &tab;
  map_f32(x, y, n, [gpu_erf, t](float v) { return gelu_one(v, gpu_erf, t); });
}

// erff_map: Shaders.lean:204-208: y[t] = bits(erff(bits^-1(base + t))), four
// consecutive patterns per thread and trip, stored as one 16-byte vector.
__global__ void g_erff_map(uint32_t base, int64_t n, uint32_t *__restrict__ y) {
  __shared__ shlo_erf::ErfSmem tab;
  shlo_erf::erf_smem_load(&tab);
  __syncthreads();
  const shlo_erf::ErfSmem *t = &tab;
  const int64_t nv = n >> 2;
  const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = t0; i < nv; i += stride) {
    const uint32_t p = base + (uint32_t)(4 * i);
    reinterpret_cast<uint4 *>(y)[i] =
        make_uint4(fbits(shlo_erf::erff_cr_smem(bitsf(p), t)), fbits(shlo_erf::erff_cr_smem(bitsf(p + 1u), t)),
                   fbits(shlo_erf::erff_cr_smem(bitsf(p + 2u), t)), fbits(shlo_erf::erff_cr_smem(bitsf(p + 3u), t)));
  }
  for (int64_t j = 4 * nv + t0; j < n; j += stride) y[j] = fbits(shlo_erf::erff_cr_smem(bitsf(base + (uint32_t)j), t));
}

// divide and sqrt: SoftFloat.lean:262-305, correctly rounded binary32 with the
// soft-float NaN rules: a NaN operand is returned quieted (the first one
// first), an invalid operation gives 0x7FC00000; sqrt returns +inf, a positive
// NaN (unquieted) and +-0 unchanged, and 0x7FC00000 for any negative input.
__device__ __forceinline__ float divide_one(float u, float v) {
  const uint32_t ub = fbits(u), vb = fbits(v);
  if ((ub & 0x7FFFFFFFu) > 0x7F800000u) return bitsf(ub | 0x00400000u);
  if ((vb & 0x7FFFFFFFu) > 0x7F800000u) return bitsf(vb | 0x00400000u);
  const float r = __fdiv_rn(u, v);
  return r != r ? bitsf(0x7FC00000u) : r;
}

__global__ void g_divide(const float *__restrict__ a, const float *__restrict__ b, float *__restrict__ y, int64_t n) {
  map2_f32(a, b, y, n, [](float u, float v) { return divide_one(u, v); });
}

__device__ __forceinline__ float sqrt_one(float u) {
  const uint32_t b = fbits(u);
  if ((b & 0x7FFFFFFFu) == 0) return u;
  if (b >> 31) return bitsf(0x7FC00000u);
  if (b >= 0x7F800000u) return u;
  return __fsqrt_rn(u);
}

__global__ void g_sqrt(const float *__restrict__ a, float *__restrict__ y, int64_t n) {
  map_f32(a, y, n, [](float u) { return sqrt_one(u); });
}

// Binary64 on uint64 bit patterns (SoftFloat.lean:137-259, Shaders.lean:231-257):
// the GPU's IEEE binary64 units, with arm64's NaN rules written out (a NaN
// operand quieted, the first one first; invalid -> 0x7FF8000000000000), floor
// exact, and the conversion to int64 truncating with saturation (NaN -> 0).
#define QNAN64 0x7FF8000000000000ull
__device__ __forceinline__ bool nan64(uint64_t v) { return (v & 0x7FFFFFFFFFFFFFFFull) > 0x7FF0000000000000ull; }

__device__ __forceinline__ uint64_t f64_one(int op, uint64_t u, uint64_t v) {
  if (op == 4)  // floor
    return nan64(u) ? (u | 0x8000000000000ull) : (uint64_t)__double_as_longlong(floor(__longlong_as_double((long long)u)));
  if (op == 5) {  // to int64, toward zero, saturating
    const double d = __longlong_as_double((long long)u);
    if (nan64(u)) return 0;
    if (d >= 9223372036854775808.0) return 0x7FFFFFFFFFFFFFFFull;
    if (d <= -9223372036854775808.0) return 0x8000000000000000ull;
    return (uint64_t)__double2ll_rz(d);
  }
  if (nan64(u)) return u | 0x8000000000000ull;
  if (nan64(v)) return v | 0x8000000000000ull;
  const double x = __longlong_as_double((long long)u), z = __longlong_as_double((long long)v);
  double q;
  switch (op) {
    case 0: q = __dadd_rn(x, z); break;
    case 1: q = __dsub_rn(x, z); break;
    case 2: q = __dmul_rn(x, z); break;
    default: q = __ddiv_rn(x, z); break;
  }
  return (q != q) ? QNAN64 : (uint64_t)__double_as_longlong(q);
}

// Two uint64 per 16-byte vector. b is read only by the binary ops (floor and
// the int64 conversion ignore it).
__global__ void g_f64_ew(const uint64_t *__restrict__ a, const uint64_t *__restrict__ b, uint64_t *__restrict__ y,
                         int64_t n, int op) {
  const int64_t nv = n >> 1;
  const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, stride = (int64_t)gridDim.x * blockDim.x;
  const bool binary = op < 4;
  for (int64_t i = t0; i < nv; i += stride) {
    const ulonglong2 u = __ldg(reinterpret_cast<const ulonglong2 *>(a) + i);
    ulonglong2 v = make_ulonglong2(0, 0);
    if (binary) v = __ldg(reinterpret_cast<const ulonglong2 *>(b) + i);
    reinterpret_cast<ulonglong2 *>(y)[i] = make_ulonglong2(f64_one(op, u.x, v.x), f64_one(op, u.y, v.y));
  }
  for (int64_t j = 2 * nv + t0; j < n; j += stride) y[j] = f64_one(op, a[j], binary ? b[j] : 0);
}

// Exact widening; a NaN keeps its payload and is not quieted (SoftFloat.lean:73-85).
__device__ __forceinline__ uint64_t f64_of_f32_one(float x) {
  const uint32_t b = fbits(x);
  if ((b & 0x7FFFFFFFu) > 0x7F800000u)
    return ((uint64_t)(b >> 31) << 63) | 0x7FF0000000000000ull | ((uint64_t)(b & 0x7FFFFFu) << 29);
  return (uint64_t)__double_as_longlong((double)x);
}

// Two elements per thread and trip: 8 bytes in, 16 bytes out, both contiguous
// across the warp.
__global__ void g_f64_of_f32(const float *__restrict__ a, uint64_t *__restrict__ y, int64_t n) {
  const int64_t nv = n >> 1;
  const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = t0; i < nv; i += stride) {
    const float2 t = __ldg(reinterpret_cast<const float2 *>(a) + i);
    reinterpret_cast<ulonglong2 *>(y)[i] = make_ulonglong2(f64_of_f32_one(t.x), f64_of_f32_one(t.y));
  }
  for (int64_t j = 2 * nv + t0; j < n; j += stride) y[j] = f64_of_f32_one(a[j]);
}

// Round to nearest even with subnormals; a NaN is quieted, payload kept (SoftFloat.lean:95-120).
__device__ __forceinline__ float f32_of_f64_one(uint64_t d) {
  if (nan64(d)) return bitsf((uint32_t)((d >> 63) << 31) | 0x7FC00000u | (uint32_t)((d & 0xFFFFFFFFFFFFFull) >> 29));
  return __double2float_rn(__longlong_as_double((long long)d));
}

__global__ void g_f32_of_f64(const uint64_t *__restrict__ a, float *__restrict__ y, int64_t n) {
  const int64_t nv = n >> 1;
  const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = t0; i < nv; i += stride) {
    const ulonglong2 u = __ldg(reinterpret_cast<const ulonglong2 *>(a) + i);
    reinterpret_cast<float2 *>(y)[i] = make_float2(f32_of_f64_one(u.x), f32_of_f64_one(u.y));
  }
  for (int64_t j = 2 * nv + t0; j < n; j += stride) y[j] = f32_of_f64_one(a[j]);
}

template <typename K, typename... Args>
static int launch_ew(Device *dev, int64_t n, K kernel, const char *what, Args... args) {
  if (n <= 0) return 0;
  kernel<<<grid_for(n, 256, dev, 16), 256, 0, dev->stream>>>(args...);
  return launch_check(what);
}

static int simple_out(Device *dev, int dt, int64_t n, Arr **o) {
  int64_t shape[1] = {n};
  return new_array(dev, (uint8_t)dt, shape, 1, o);
}

int k_silu(Device *dev, Arr *x, const uint32_t *p, Arr **out) {
  int64_t n = p[0];
  SHLO_TRY(require_dtype(x, kF32, "silu") || check_elems(x, n, "silu"));
  Arr *o;
  SHLO_TRY(simple_out(dev, kF32, n, &o));
  if (launch_ew(dev, n, g_silu, "silu", (const float *)data_ptr(x), (float *)o->buf->ptr, n, (int)(p[1] != 0))) {
    shlo_release(o);
    return 1;
  }
  *out = o;
  return 0;
}

int k_gelu_erf(Device *dev, Arr *x, const uint32_t *p, Arr **out) {
  int64_t n = p[0];
  SHLO_TRY(require_dtype(x, kF32, "gelu_erf") || check_elems(x, n, "gelu_erf"));
  if (current_flavor() == 1 && p[1] == 0)
    return fail("gelu_erf: the stock build's erff is Apple libsystem_m's platform erff, which is not carried "
                "(this backend carries the correctly rounded erff of the pinned build)");
  Arr *o;
  SHLO_TRY(simple_out(dev, kF32, n, &o));
  if (launch_ew(dev, n, g_gelu_erf, "gelu_erf", (const float *)data_ptr(x), (float *)o->buf->ptr, n, (int)(p[1] != 0))) {
    shlo_release(o);
    return 1;
  }
  *out = o;
  return 0;
}

int k_erff_map(Device *dev, const uint32_t *p, Arr **out) {
  int64_t n = p[1];
  Arr *o;
  SHLO_TRY(simple_out(dev, kU32, n, &o));
  if (launch_ew(dev, n, g_erff_map, "erff_map", p[0], n, (uint32_t *)o->buf->ptr)) {
    shlo_release(o);
    return 1;
  }
  *out = o;
  return 0;
}

int k_divide(Device *dev, Arr *a, Arr *b, const uint32_t *p, Arr **out) {
  int64_t n = p[0];
  SHLO_TRY(require_dtype(a, kF32, "divide") || require_dtype(b, kF32, "divide"));
  SHLO_TRY(check_elems(a, n, "divide") || check_elems(b, n, "divide"));
  Arr *o;
  SHLO_TRY(simple_out(dev, kF32, n, &o));
  if (launch_ew(dev, n, g_divide, "divide", (const float *)data_ptr(a), (const float *)data_ptr(b),
                (float *)o->buf->ptr, n)) {
    shlo_release(o);
    return 1;
  }
  *out = o;
  return 0;
}

int k_sqrt(Device *dev, Arr *a, const uint32_t *p, Arr **out) {
  int64_t n = p[0];
  SHLO_TRY(require_dtype(a, kF32, "sqrt") || check_elems(a, n, "sqrt"));
  Arr *o;
  SHLO_TRY(simple_out(dev, kF32, n, &o));
  if (launch_ew(dev, n, g_sqrt, "sqrt", (const float *)data_ptr(a), (float *)o->buf->ptr, n)) {
    shlo_release(o);
    return 1;
  }
  *out = o;
  return 0;
}

int k_f64_ew(Device *dev, Arr *a, Arr *b, const uint32_t *p, Arr **out) {
  int64_t n = p[0];
  int op = (int)p[1];
  if (op < 0 || op > 5) return fail("f64_ew: op %d not carried", op);
  SHLO_TRY(require_dtype(a, kU64, "f64_ew") || require_dtype(b, kU64, "f64_ew"));
  SHLO_TRY(check_elems(a, n, "f64_ew") || check_elems(b, n, "f64_ew"));
  Arr *o;
  SHLO_TRY(simple_out(dev, kU64, n, &o));
  if (launch_ew(dev, n, g_f64_ew, "f64_ew", (const uint64_t *)data_ptr(a), (const uint64_t *)data_ptr(b),
                (uint64_t *)o->buf->ptr, n, op)) {
    shlo_release(o);
    return 1;
  }
  *out = o;
  return 0;
}

int k_f64_of_f32(Device *dev, Arr *a, const uint32_t *p, Arr **out) {
  int64_t n = p[0];
  SHLO_TRY(require_dtype(a, kF32, "f64_of_f32") || check_elems(a, n, "f64_of_f32"));
  Arr *o;
  SHLO_TRY(simple_out(dev, kU64, n, &o));
  if (launch_ew(dev, n, g_f64_of_f32, "f64_of_f32", (const float *)data_ptr(a), (uint64_t *)o->buf->ptr, n)) {
    shlo_release(o);
    return 1;
  }
  *out = o;
  return 0;
}

int k_f32_of_f64(Device *dev, Arr *a, const uint32_t *p, Arr **out) {
  int64_t n = p[0];
  SHLO_TRY(require_dtype(a, kU64, "f32_of_f64") || check_elems(a, n, "f32_of_f64"));
  Arr *o;
  SHLO_TRY(simple_out(dev, kF32, n, &o));
  if (launch_ew(dev, n, g_f32_of_f64, "f32_of_f64", (const uint64_t *)data_ptr(a), (float *)o->buf->ptr, n)) {
    shlo_release(o);
    return 1;
  }
  *out = o;
  return 0;
}

}  // namespace shlo

// ================================================= mul_mat without allocation ====
// Some callers cannot let this library allocate device memory: a host runtime
// whose device memory is all owned by its own allocator (a framework's caching
// pool, a fixed arena), or one that must not allocate while it records work.
// shlo_mul_mat_noalloc serves them: the caller passes the operands and the
// output as device pointers, and the two packed operands of the fast path go to
// the fixed scratch array below instead of to allocated storage. The array is
// part of the library image: every GPU that loads the library holds it until
// the process exits.

namespace shlo {

constexpr size_t kNoAllocScratchBytes = (size_t)16 << 20;  // 16 MiB
static __device__ __align__(256) float g_mm_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

// The scratch array's device address, looked up once per device with that device
// current (in host code the array's name is only a host-side stand-in).
static std::mutex g_noalloc_mu;
static float *g_noalloc_ptr[64];

static int noalloc_scratch(int dev, float **out) {
  if (dev < 0 || dev >= 64) return fail("mul_mat_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_mm_noalloc_scratch);
    if (e != cudaSuccess) return cuda_check(e, "mul_mat_noalloc: scratch address");
    g_noalloc_ptr[dev] = (float *)p;
  }
  *out = g_noalloc_ptr[dev];
  return 0;
}

}  // namespace shlo

extern "C" int shlo_mul_mat_noalloc(const float *w, const float *x, float *y, int64_t K, int64_t M, int64_t R,
                                    int64_t N, int64_t w_batch_stride, void *stream) {
  using namespace shlo;
  cudaStream_t s = (cudaStream_t)stream;
  if (!w || !x || !y) return fail("mul_mat_noalloc: null pointer");
  if (K <= 0 || M <= 0 || R < 0 || N <= 0 || R % N)
    return fail("mul_mat_noalloc: K=%lld M=%lld R=%lld N=%lld not carried", (long long)K, (long long)M, (long long)R,
                (long long)N);
  const int64_t wbs = w_batch_stride;
  if (wbs && wbs < M * K) return fail("mul_mat_noalloc: w batch stride %lld below M*K", (long long)wbs);
  if (K > INT32_MAX || M > INT32_MAX) return fail("mul_mat_noalloc: K or M too large");
  if (R * M == 0) return 0;
  int devid = 0;
  SHLO_CUDA(cudaGetDevice(&devid));
  const int flavor = current_flavor();
  const int64_t np = K & ~(int64_t)15;
  if (np < 16) {  // all tail: the one-output-per-thread kernel needs no scratch
    int sms = 0;
    SHLO_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, devid));
    int64_t blocks = (R * M + 255) / 256;
    if (blocks > (int64_t)sms * 8) blocks = (int64_t)sms * 8;
    k_mul_mat_naive<<<(unsigned)blocks, 256, 0, s>>>(w, x, y, (int)K, (int)M, R, N, wbs, 0, flavor);
    return launch_check("mul_mat_noalloc");
  }
  const int64_t nb = R / N;
  const int seg = (int)(np / 16);
  const int segp = (seg + 3) & ~3;
  const int Mp = (int)((M + mm::BM - 1) / mm::BM * mm::BM);
  const int64_t Bx = wbs ? nb : 1;
  const int64_t Nx = wbs ? N : R;
  const int Np = (int)((Nx + mm::BN - 1) / mm::BN * mm::BN);
  const int64_t Wb = wbs ? nb : 1;
  const int64_t w_floats = Wb * 16 * segp * (int64_t)Mp;
  const int64_t x_floats = Bx * 16 * segp * (int64_t)Np;
  const int64_t need = (w_floats + x_floats) * (int64_t)sizeof(float);
  if (need > (int64_t)kNoAllocScratchBytes)
    return fail("mul_mat_noalloc: the packed operands need %lld bytes of scratch, above the %zu-byte maximum of this "
                "entry point (use the allocating kernel for larger shapes)", (long long)need, kNoAllocScratchBytes);
  float *scratch;
  SHLO_TRY(noalloc_scratch(devid, &scratch));
  // Both packed regions are written in full by the pack kernels (padding
  // included), so nothing in the scratch array has to start at zero.
  float *wp = scratch, *xp = scratch + w_floats;
  launch_pack(w, (int)M, (int)K, wbs, (int)Wb, seg, segp, Mp, -0.0f, wp, s);
  SHLO_TRY(launch_check("mul_mat_noalloc pack"));
  launch_pack(x, (int)Nx, (int)K, Nx * K, (int)Bx, seg, segp, Np, 0.0f, xp, s);
  SHLO_TRY(launch_check("mul_mat_noalloc pack"));
  MMArgs a;
  a.wp = wp;
  a.xp = xp;
  a.w = w;
  a.x = x;
  a.y = y;
  a.K = (int)K;
  a.M = (int)M;
  a.np = (int)np;
  a.segp = segp;
  a.Mp = Mp;
  a.Np = Np;
  a.Nx = Nx;
  a.wbs = wbs;
  a.r_tiles = Np / mm::BN;
  a.flavor = flavor;
  const size_t smem = (size_t)mm::NS * mm::STAGE_FLOATS * sizeof(float);
  SHLO_CUDA(cudaFuncSetAttribute(k_mul_mat_fast, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid(Mp / mm::BM, (unsigned)(Bx * a.r_tiles));
  k_mul_mat_fast<<<grid, mm::THREADS, smem, s>>>(a);
  return launch_check("mul_mat_noalloc");
}
