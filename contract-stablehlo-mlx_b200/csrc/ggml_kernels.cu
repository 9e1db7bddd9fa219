// The exact kernels: ggml-cpu's arm64 arithmetic, bit for bit, on sm_100a.
//
// Each kernel reproduces the reference's Lean kernel spec
// (StablehloMlx/Kernels/Shaders.lean) with the parameter words of
// StablehloMlx/Kernels/Run.lean:62-104. Built with -fmad=false: every fused
// multiply-add below is an explicit __fmaf_rn where ggml uses vfmaq_f32, and
// every other product and sum is rounded on its own.
#include <atomic>
#include <cmath>

#include "common.cuh"
#include <utility>

#include "erff_cr.cuh"
#include "gelu.cuh"
#include "ggml_math.cuh"
#include "mul_mat.cuh"

namespace shlo {

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
// The packed-segment order of ggml_vec_dot_f32, the operand layout and the
// TMEM-stack and register-stack kernels are in mul_mat.cuh; here are the
// reference's one-thread-per-output form, the operand pack, the noalloc
// entry's kernel and the host dispatch.
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

// $SHLO_MUL_MAT_PATH = naive | fast forces one of the two exact paths (both give
// the same bits; the tests run each); unset, the size decides.
static int mm_path() {
  const char *e = getenv("SHLO_MUL_MAT_PATH");
  if (e && !strcmp(e, "naive")) return 1;
  if (e && !strcmp(e, "fast")) return 2;
  if (e && !strcmp(e, "seg")) return 3;
  return 0;
}

// A 2-D tensor map of a packed operand ([outer][inner] floats, rows of `inner`),
// box box_inner x 16 rows, no swizzle, zero fill outside (never reached: the
// packed operands are padded to whole tiles). cuTensorMapEncodeTiled is reached
// through the runtime, so the library links no driver library.
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static int tensor_map_2d(CUtensorMap *map, const float *base, uint64_t inner, uint64_t outer, uint32_t box_inner) {
  static const EncodeTiledFn fn = [] {
    void *f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<EncodeTiledFn>(f);
  }();
  if (!fn) return fail("mul_mat: the driver's cuTensorMapEncodeTiled is not available");
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {inner * sizeof(float)};
  const cuuint32_t box[2] = {box_inner, (cuuint32_t)mt::BK};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail("mul_mat: tensor map of %llu x %llu floats (box %u x %d): driver error %d", (unsigned long long)outer,
                (unsigned long long)inner, box_inner, mt::BK, (int)r);
  return 0;
}

static int pack_operand(Device *dev, const float *src, int rows, int K, int64_t src_batch, int batches, int seg,
                        int segp, int rows_p, float pad, Buffer **out) {
  // k_mm_pack writes whole blocks of 64 rows
  if (rows_p % 64) return fail("mul_mat pack: %d padded rows, not a multiple of 64", rows_p);
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

// The packed x of a product of K x M over R rows (one weight, N = R): its
// segments and padded rows, as mul_mat_ep would make them (the same choice of
// kernel). False where the product packs no x (the one-thread-an-output path)
// or its x needs segment padding or a tail (K not a multiple of 64): such an x
// cannot be handed over packed.
bool mm_packed_x_layout(int64_t K, int64_t M, int64_t R, int *segp, int *Np) {
  const int path = mm_path();
  if (K % 64 || K < 64 || R <= 0 || M <= 0) return false;
  if (!(path >= 2 || (path == 0 && R * M >= 4096))) return false;
  const int seg = (int)(K / 16);
  const bool short_k = path != 3 && (seg == 4 || (M <= 64 && seg <= 16));
  const bool seg_k = path == 3 || (path == 0 && !short_k && R * M <= ((int64_t)1 << 21));
  const int WM = M <= 64 ? 1 : 2;
  const int BN = seg_k ? sg::TR : short_k ? ms::BN : WM == 1 ? mt::Tile<1>::BN : mt::Tile<2>::BN;
  const int PN = BN < 64 ? 64 : BN;
  *segp = seg;
  *Np = (int)((R + PN - 1) / PN * PN);
  return true;
}

// The product with its fused epilogue. *gelu_done (when EP_GELU is asked for)
// is set when k_mul_mat_tm ran gelu_erf in its epilogue; the other paths leave
// it to the caller. x_np > 0: x's storage already holds this product's packed
// x (mm_packed_x_layout's, x_np rows). y_pack = {segp, Np}: the result is for a
// product that takes it packed; *pack_done is set when the epilogue wrote it in
// that layout (k_mul_mat_tm with gelu_erf), and the result's storage is sized
// for it either way.
static int mul_mat_ep(Device *dev, Arr *w, Arr *x, const uint32_t *p, Arr *bias, Arr *res, int ep, Arr **out,
                      bool *gelu_done, int x_np = 0, const int *y_pack = nullptr, bool *pack_done = nullptr) {
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
  int64_t shape[1] = {y_pack ? M * (int64_t)y_pack[1] : R * M};
  Arr *o;
  SHLO_TRY(new_array(dev, kF32, shape, 1, &o));
  o->shape[0] = R * M;  // (a packed result's storage holds its padded rows too)
  const int flavor = current_flavor();
  const int64_t np = K & ~(int64_t)15;
  int path = mm_path();
  bool fast = !plain && np >= 16 && (path >= 2 || (path == 0 && R * M >= 4096));
  if (R * M == 0) {
    *out = o;
    return 0;
  }
  if (!fast && x_np) {
    shlo_release(o);
    return fail("mul_mat: a packed x handed to the one-thread-an-output path");
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
  const int64_t Bx = wbs ? nb : 1;
  const int64_t Nx = wbs ? N : R;
  // k_mul_mat_seg (32 x 32 tiles, the sixteen chains side by side in a CTA):
  // products of up to 2^21 outputs, where 128 x 128 tiles would leave most of
  // the GPU idle; $SHLO_MUL_MAT_PATH=seg forces it.
  const bool short_k = path != 3 && (segp == 4 || (M <= 64 && segp <= 16));
  const bool seg_k = path == 3 || (path == 0 && !short_k && Bx * Nx * M <= ((int64_t)1 << 21));
  const int WM = M <= 64 ? 1 : 2;
  const int BM = seg_k ? sg::TM : short_k ? ms::BM : WM == 1 ? mt::Tile<1>::BM : mt::Tile<2>::BM;
  const int BN = seg_k ? sg::TR : short_k ? ms::BN : WM == 1 ? mt::Tile<1>::BN : mt::Tile<2>::BN;
  // padded to whole tiles, and to the pack's blocks of 64 rows
  const int PM = BM < 64 ? 64 : BM, PN = BN < 64 ? 64 : BN;
  const int Mp = (int)((M + PM - 1) / PM * PM);
  const int Np = (int)((Nx + PN - 1) / PN * PN);
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
  if (x_np) {
    // x is this product's packed x already (the producer wrote it so)
    if (K % 64 || segp != seg || Bx != 1 || Np != x_np || !x->buf || x->offset ||
        x->buf->bytes < (size_t)16 * segp * Np * sizeof(float)) {
      buffer_release(wpk);
      shlo_release(o);
      return fail("mul_mat: a packed x that does not match this product's layout");
    }
    xpk = x->buf;
    buffer_retain(xpk);
  } else if (pack_operand(dev, (const float *)data_ptr(x), (int)Nx, (int)K, Nx * K, (int)Bx, seg, segp, Np, 0.0f,
                          &xpk)) {
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
  if (seg_k || short_k) {
    const unsigned grid = (unsigned)((int64_t)(Mp / BM) * Bx * a.r_tiles);
    if (seg_k)
      launch_mul_mat_seg(ep != 0, grid, dev->stream, a);
    else
      launch_mul_mat_short(segp / 4, ep != 0, grid, dev->stream, a);
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
  static bool attr_done[64] = {false};
  if (!attr_done[dev->id]) {
    const int rc = cuda_check(mul_mat_tm_attributes<1>(), "mul_mat attribute") ||
         cuda_check(mul_mat_tm_attributes<2>(), "mul_mat attribute") ||
         cuda_check(mul_mat_tm_attributes<4>(), "mul_mat attribute") ||
         cuda_check(mul_mat_tm_attributes<8>(), "mul_mat attribute") ||
         cuda_check(mul_mat_tm_attributes<16>(), "mul_mat attribute");
    if (rc) {
      buffer_release(wpk);
      buffer_release(xpk);
      shlo_release(o);
      return 1;
    }
    attr_done[dev->id] = true;
  }
  // A tile's fold tree split over SPLIT CTAs (each a subtree; the last to
  // arrive adds the top levels). $SHLO_MM_SPLIT = 1 | 2 | 4 forces one form;
  // all give the same bits.
  const int64_t tiles = (int64_t)(Mp / BM) * Bx * a.r_tiles;
  const int64_t slots = (int64_t)mt::CTAS_PER_SM * dev->sm_count;
  auto wave_fill = [&](int64_t t) { return (double)t / (double)(((t + slots - 1) / slots) * slots); };
  // Halves where measured faster (B200, the denoiser's shapes): long K
  // (>= 2048) or narrow M (<= 512), each half at least 16 stages of 16 k, the
  // grid no fuller in its last wave than halved, and fewer than four waves of
  // tiles (with more, one CTA a tile measured as fast or faster: the output
  // projection at 131072 rows 44.7 against 43.5 TFLOP/s). Smaller splits for
  // tiny grids (below).
  int split = 1;
  if (segp / 2 >= 16 && (segp >= 128 || M <= 512) && tiles < 4 * slots &&
      wave_fill(2 * tiles) + 0.01 >= wave_fill(tiles))
    split = 2;
  // A grid of a few tiles (the timestep MLP, BASELINE config 1, a batch of one)
  // leaves most SMs idle: quarters, eighths or sixteenths of the tree make each
  // CTA's K that much shorter, as long as the grid stays within one CTA an SM
  // and every CTA keeps whole stages of 16 packed k (2 or 1 segments a CTA:
  // segp a multiple of 8 or 16).
  auto valid = [&](int s) { return s <= 4 ? segp % 4 == 0 : segp % s == 0; };
  if (4 * tiles <= slots / 2 && segp >= 8) split = 4;
  if (split == 4 && 8 * tiles <= slots / 2 && valid(8)) split = 8;
  if (split == 8 && 16 * tiles <= slots / 2 && valid(16)) split = 16;
  if (const char *e = getenv("SHLO_MM_SPLIT")) {
    // a forced form; the largest valid one at or below it
    split = 1;
    for (int s : {2, 4, 8, 16})
      if (s <= atoi(e) && valid(s)) split = s;
  }
  const bool shared_tile = split > 1;
  const unsigned grid = (unsigned)(split * tiles);
  Buffer *park, *ctr = nullptr;
  if (buffer_alloc(dev, (size_t)grid * mt::THREADS * 64 * sizeof(float), &park) ||
      (shared_tile && buffer_alloc(dev, (size_t)tiles * sizeof(int), &ctr)) ||
      (shared_tile && cuda_check(cudaMemsetAsync(ctr->ptr, 0, (size_t)tiles * sizeof(int), dev->stream), "mul_mat counters"))) {
    buffer_release(park);
    buffer_release(ctr);
    buffer_release(wpk);
    buffer_release(xpk);
    shlo_release(o);
    return 1;
  }
  a.park = (float *)park->ptr;
  a.ctr = shared_tile ? (int *)ctr->ptr : nullptr;
  a.err = dev->pipe_err_dev;
  CUtensorMap tw, tx;
  if (tensor_map_2d(&tw, a.wp, (uint64_t)Mp, (uint64_t)Wb * 16 * segp, (uint32_t)BM) ||
      tensor_map_2d(&tx, a.xp, (uint64_t)Np, (uint64_t)Bx * 16 * segp, (uint32_t)BN)) {
    buffer_release(park);
    buffer_release(ctr);
    buffer_release(wpk);
    buffer_release(xpk);
    shlo_release(o);
    return 1;
  }
  const bool stage_fold = segp % 16 == 0;
  int epi = ep != 0;
  if ((ep & EP_GELU) && WM == 2) {
    epi = 2;
    *gelu_done = true;
    if (y_pack && y_pack[1] == Np && 16 * (int64_t)y_pack[0] == M && Bx == 1) {
      a.ypk_segp = y_pack[0];
      a.ypk_np = y_pack[1];
      *pack_done = true;
    }
  }
  if (split == 16) launch_mul_mat_tm<16>(WM, stage_fold, epi, grid, dev->stream, a, tw, tx);
  else if (split == 8) launch_mul_mat_tm<8>(WM, stage_fold, epi, grid, dev->stream, a, tw, tx);
  else if (split == 4) launch_mul_mat_tm<4>(WM, stage_fold, epi, grid, dev->stream, a, tw, tx);
  else if (split == 2) launch_mul_mat_tm<2>(WM, stage_fold, epi, grid, dev->stream, a, tw, tx);
  else launch_mul_mat_tm<1>(WM, stage_fold, epi, grid, dev->stream, a, tw, tx);
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
    // With the row in registers (G > 0), the group sums' binades: when every
    // partial sum of them is exact in binary64 (see exact_sum), the lanes add
    // their own parts and a shuffle tree replaces lane 0's chain.
    int pmin = 255, pmax = 0;
    bool pspecial = false;
    double psum = 0.0;
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
          const float part = __fadd_rn(__fadd_rn(e.x, e.y), __fadd_rn(e.z, e.w));
          parts[lane + 32 * i] = (double)part;
          if (G > 0) {
            const uint32_t pb = fbits(part) & 0x7FFFFFFFu;
            const int pe = (int)(pb >> 23);
            pspecial |= pe == 255;
            if (pb) {
              pmin = min(pmin, pe ? pe : 1);
              pmax = max(pmax, pe ? pe : 1);
            }
            psum = __dadd_rn(psum, (double)part);
          }
        }
      }
      __syncwarp();
      // Nonzero terms with exponent fields in [pmin, pmax] are multiples of
      // 2^(pmin - 150) below 2^(pmax - 126); ng of them sum, in any order, to
      // multiples of 2^(pmin - 150) below 2^(pmax - 126 + ceil(log2 ng)), all
      // exact in binary64 when pmax - pmin + 24 + ceil(log2 ng) <= 53. (G > 0:
      // one chunk holds the whole row. Not for the planted float chain.)
      bool exact = false;
      if (G > 0) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          pmin = min(pmin, __shfl_xor_sync(0xffffffffu, pmin, o));
          pmax = max(pmax, __shfl_xor_sync(0xffffffffu, pmax, o));
          psum = __dadd_rn(psum, __shfl_xor_sync(0xffffffffu, psum, o));
        }
        const int lg = ng > 1 ? 32 - __clz(ng - 1) : 0;
        exact = !float_sum && !__any_sync(0xffffffffu, pspecial) && (pmin > pmax || pmax - pmin + 24 + lg <= 53);
        if (exact) sum = psum;
      }
      if (lane == 0 && !exact) {
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


static const char kGeluStockRefusal[] =
    "gelu_erf: the stock build's erff is Apple libsystem_m's platform erff, which is not carried "
    "(this backend carries the correctly rounded erff of the pinned build)";

int k_mul_mat_fused(Device *dev, Arr *w, Arr *x, const uint32_t *p, Arr *bias, Arr *res, int ep, int x_np,
                    const int *y_pack, Arr **out) {
  if ((ep & EP_GELU) && current_flavor() == 1) return fail("%s", kGeluStockRefusal);
  bool gelu_done = false, pack_done = false;
  Arr *o;
  SHLO_TRY(mul_mat_ep(dev, w, x, p, bias, res, ep, &o, &gelu_done, x_np, y_pack, &pack_done));
  const int64_t R = p[2], M = p[1];
  if ((ep & EP_GELU) && !gelu_done) {
    // The product (with its adds) by a kernel without the gelu epilogue: the
    // gelu_erf kernel on its result, the same bits.
    const uint32_t gp[2] = {(uint32_t)(R * M), 0};
    Arr *g;
    const int rc = k_gelu_erf(dev, o, gp, &g);
    shlo_release(o);
    SHLO_TRY(rc);
    o = g;
  }
  if (y_pack && !pack_done) {
    Arr *q;
    const int rc = k_pack_x(dev, o, R, M, y_pack, &q);
    shlo_release(o);
    SHLO_TRY(rc);
    o = q;
  }
  *out = o;
  return 0;
}

int k_pack_x(Device *dev, Arr *src, int64_t rows, int64_t K, const int *y_pack, Arr **out) {
  if (K % 64 || 16 * (int64_t)y_pack[0] != K || y_pack[1] < rows || y_pack[1] % 64 || numel(src) < rows * K ||
      ((uintptr_t)data_ptr(src) & 15))
    return fail("pack: a %lld x %lld operand does not fit the packed layout (%d, %d)", (long long)rows, (long long)K,
                y_pack[0], y_pack[1]);
  int64_t shape[1] = {K * (int64_t)y_pack[1]};
  Arr *q;
  SHLO_TRY(new_array(dev, kF32, shape, 1, &q));
  q->shape[0] = rows * K;  // (the storage holds the padded rows too)
  launch_pack((const float *)data_ptr(src), (int)rows, (int)K, rows * K, 1, (int)(K / 16), y_pack[0], y_pack[1], 0.0f,
              (float *)q->buf->ptr, dev->stream);
  if (launch_check("pack")) {
    shlo_release(q);
    return 1;
  }
  *out = q;
  return 0;
}

int k_mul_mat_ep(Device *dev, Arr *w, Arr *x, const uint32_t *p, Arr *bias, Arr *res, int ep, Arr **out) {
  return k_mul_mat_fused(dev, w, x, p, bias, res, ep, 0, nullptr, out);
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

// One warp a row, for rows of 128 c (c <= 8) values held in registers: lane l
// holds the four-value groups l, l + 32, ..., so each 16-byte load is a group.
// Each binary64 sum (the values; then the group sums) is reassociated only when
// no partial sum can round: nonzero binary32 terms whose exponent fields lie in
// [emin, emax] are multiples of 2^(emin - 150) below 2^(emax - 126), so n of
// them, in any order, stay multiples of 2^(emin - 150) below
// 2^(emax - 126 + ceil(log2 n)), exact in binary64 when emax - emin + 24 +
// ceil(log2 n) <= 53; then the lanes add their own terms and a shuffle tree
// gives the spec's sum. Otherwise (or with an infinity or NaN) the row goes to
// the warp's shared-memory buffer and lane 0 runs the spec's serial chain.
// Every warp collective sits outside the per-row branches.
//
// norm_row: one row (a warp), the norm (and the fused affine) of row `row` into
// res, lane l holding the float4 groups l, l + 32, ...; rowbuf: the warp's N
// floats for the serial chains.
template <int C>
__device__ __forceinline__ void norm_row(const float *__restrict__ x, int64_t row, float eps,
                                         const float *__restrict__ gamma, const float *__restrict__ beta,
                                         float *rowbuf, int lane, float4 (&res)[C]) {
  constexpr int N = 128 * C;
  const int lg_n = 32 - __clz(N - 1), lg_g = 32 - __clz(N / 4 - 1);
  auto span = [&](float v, int &lo, int &hi, bool &sp) {
    const uint32_t b = fbits(v) & 0x7FFFFFFFu;
    const int e = (int)(b >> 23);
    sp |= e == 255;
    if (b) {
      lo = min(lo, e ? e : 1);
      hi = max(hi, e ? e : 1);
    }
  };
  auto exact = [&](int lo, int hi, bool sp, int lg) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
      hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, o));
    }
    return !__any_sync(0xffffffffu, sp) && (lo > hi || hi - lo + 24 + lg <= 53);
  };
  const float4 *xr = reinterpret_cast<const float4 *>(x + row * N);
  float4 v[C];
#pragma unroll
  for (int c = 0; c < C; c++) v[c] = __ldg(xr + lane + 32 * c);
  // the row sum
  int lo = 255, hi = 0;
  bool sp = false;
  double sum = 0.0;
#pragma unroll
  for (int c = 0; c < C; c++) {
    span(v[c].x, lo, hi, sp); span(v[c].y, lo, hi, sp); span(v[c].z, lo, hi, sp); span(v[c].w, lo, hi, sp);
    sum = __dadd_rn(__dadd_rn(__dadd_rn(__dadd_rn(sum, (double)v[c].x), (double)v[c].y), (double)v[c].z),
                    (double)v[c].w);
  }
  const bool ex1 = exact(lo, hi, sp, lg_n);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum = __dadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
  if (!ex1) {  // warp-uniform
#pragma unroll
    for (int c = 0; c < C; c++) reinterpret_cast<float4 *>(rowbuf)[lane + 32 * c] = v[c];
    __syncwarp();
    if (lane == 0) {
      double s0 = 0.0;
      for (int k = 0; k < N; k += 8) {  // eight values loaded ahead of their serial adds
        double t[8];
#pragma unroll
        for (int i = 0; i < 8; i++) t[i] = (double)rowbuf[k + i];
#pragma unroll
        for (int i = 0; i < 8; i++) s0 = __dadd_rn(s0, t[i]);
      }
      sum = s0;
    }
    sum = __shfl_sync(0xffffffffu, sum, 0);
    __syncwarp();
  }
  const float mean = __fdiv_rn(__double2float_rn(sum), (float)N);
  // the group sums of squared deviations
  float q[C];
  lo = 255; hi = 0; sp = false;
  double s2 = 0.0;
#pragma unroll
  for (int c = 0; c < C; c++) {
    const float d0 = __fsub_rn(v[c].x, mean), d1 = __fsub_rn(v[c].y, mean);
    const float d2 = __fsub_rn(v[c].z, mean), d3 = __fsub_rn(v[c].w, mean);
    q[c] = __fadd_rn(__fadd_rn(__fmul_rn(d0, d0), __fmul_rn(d1, d1)), __fadd_rn(__fmul_rn(d2, d2), __fmul_rn(d3, d3)));
    span(q[c], lo, hi, sp);
    s2 = __dadd_rn(s2, (double)q[c]);
  }
  const bool ex2 = exact(lo, hi, sp, lg_g);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s2 = __dadd_rn(s2, __shfl_xor_sync(0xffffffffu, s2, o));
  if (!ex2) {  // warp-uniform: the group sums in group order
#pragma unroll
    for (int c = 0; c < C; c++) rowbuf[lane + 32 * c] = q[c];
    __syncwarp();
    if (lane == 0) {
      double t2 = 0.0;
      for (int k = 0; k < N / 4; k += 8) {
        double t[8];
#pragma unroll
        for (int i = 0; i < 8; i++) t[i] = (double)rowbuf[k + i];
#pragma unroll
        for (int i = 0; i < 8; i++) t2 = __dadd_rn(t2, t[i]);
      }
      s2 = t2;
    }
    s2 = __shfl_sync(0xffffffffu, s2, 0);
    __syncwarp();
  }
  const float var = __double2float_rn(__ddiv_rn(s2, (double)N));
  const float scl = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
#pragma unroll
  for (int c = 0; c < C; c++) {
    res[c].x = arm_nan(__fmul_rn(__fsub_rn(v[c].x, mean), scl));
    res[c].y = arm_nan(__fmul_rn(__fsub_rn(v[c].y, mean), scl));
    res[c].z = arm_nan(__fmul_rn(__fsub_rn(v[c].z, mean), scl));
    res[c].w = arm_nan(__fmul_rn(__fsub_rn(v[c].w, mean), scl));
    if (gamma) {  // the executor's fused affine: (y * gamma) + beta, each rounded alone
      const float4 g = __ldg(reinterpret_cast<const float4 *>(gamma) + lane + 32 * c);
      const float4 b = __ldg(reinterpret_cast<const float4 *>(beta) + lane + 32 * c);
      res[c] = make_float4(__fadd_rn(__fmul_rn(res[c].x, g.x), b.x), __fadd_rn(__fmul_rn(res[c].y, g.y), b.y),
                         __fadd_rn(__fmul_rn(res[c].z, g.z), b.z), __fadd_rn(__fmul_rn(res[c].w, g.w), b.w));
    }
  }
}

template <int C>  // float4 groups a lane: ncols = 128 C
__global__ void __launch_bounds__(128) g_norm_warp(const float *__restrict__ x, float *__restrict__ y, int64_t rows,
                                                   float eps, const float *__restrict__ gamma,
                                                   const float *__restrict__ beta) {
  constexpr int N = 128 * C;
  __shared__ float buf[4][N];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int64_t row = (int64_t)blockIdx.x * 4 + w; row < rows; row += (int64_t)gridDim.x * 4) {
    float4 o[C];
    norm_row<C>(x, row, eps, gamma, beta, buf[w], lane, o);
    float4 *yr = reinterpret_cast<float4 *>(y + row * N);
#pragma unroll
    for (int c = 0; c < C; c++) yr[lane + 32 * c] = o[c];
  }
}

// g_norm_warp writing its result as the packed x of a next product whose K is
// N (segments of segp = N / 16 packed k, rows_p rows: (row r, column k) at
// (leaf_of_class(k % 16) * segp + k / 16) * rows_p + r; the rows past `rows`
// zero). 8 rows at a time, one a warp, through shared memory ([8][N + 4]);
// then thread t the row t % 8 of the columns t / 8, t / 8 + 32, ... (32-byte
// stores, a warp four columns; the tile's reads spread over all 32 banks).
template <int C>
__global__ void __launch_bounds__(256) g_norm_warp_pk(const float *__restrict__ x, float *__restrict__ y, int64_t rows,
                                                      int64_t rows_p, float eps, const float *__restrict__ gamma,
                                                      const float *__restrict__ beta) {
  constexpr int N = 128 * C, TS = N + 4, segp = N / 16;
  extern __shared__ __align__(16) float sm[];  // the tile [8][TS], then the warps' row buffers [8][N]
  float *tile = sm, *buf = sm + 8 * TS;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, i = threadIdx.x & 7;
  for (int64_t r0 = (int64_t)blockIdx.x * 8; r0 < rows_p; r0 += (int64_t)gridDim.x * 8) {
    if (r0 + w < rows) {
      float4 o[C];
      norm_row<C>(x, r0 + w, eps, gamma, beta, buf + w * N, lane, o);
#pragma unroll
      for (int c = 0; c < C; c++) reinterpret_cast<float4 *>(tile + w * TS)[lane + 32 * c] = o[c];
    }
    __syncthreads();
    const bool live = r0 + i < rows;
#pragma unroll 4
    for (int k = threadIdx.x >> 3; k < N; k += 32)
      y[((int64_t)leaf_of_class(k & 15) * segp + (k >> 4)) * rows_p + r0 + i] = live ? tile[i * TS + k] : 0.0f;
    __syncthreads();
  }
}

int k_norm(Device *dev, Arr *x, const uint32_t *p, Arr **out) { return k_norm_affine(dev, x, p, nullptr, nullptr, out); }

int k_norm_affine(Device *dev, Arr *x, const uint32_t *p, Arr *gamma, Arr *beta, Arr **out) {
  return k_norm_affine_packed(dev, x, p, gamma, beta, nullptr, out);
}

int k_norm_affine_packed(Device *dev, Arr *x, const uint32_t *p, Arr *gamma, Arr *beta, const int *y_pack,
                         Arr **out) {
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
  const size_t smem = (size_t)NORM_ROWS * (ncols + 1) * sizeof(float);
  const bool aligned = (((uintptr_t)data_ptr(x)) & 15) == 0 &&
                       (!affine || ((((uintptr_t)gp) | ((uintptr_t)bp)) & 15) == 0);
  const bool warp_rows = ncols * rows > 0 && p[3] == 0 && ncols % 128 == 0 && ncols <= 1024 && aligned;
  // y_pack: the packed x of a next product (K = ncols), written by
  // g_norm_warp_pk, or by the pack kernel after the norm
  if (y_pack && (ncols % 64 || 16 * (int64_t)y_pack[0] != ncols || y_pack[1] < rows || y_pack[1] % 64))
    return fail("norm: a %lld x %lld result does not fit the packed layout (%d, %d)", (long long)rows,
                (long long)ncols, y_pack[0], y_pack[1]);
  if (y_pack && warp_rows) {
    int64_t shape[1] = {ncols * (int64_t)y_pack[1]};
    Arr *o;
    SHLO_TRY(new_array(dev, kF32, shape, 1, &o));
    o->shape[0] = ncols * rows;
    const size_t tbytes = (size_t)8 * (2 * ncols + 4) * sizeof(float);
    static bool attr_pk[64] = {false};
    if (!attr_pk[dev->id]) {
      int rc = 0;
      rc |= cuda_check(cudaFuncSetAttribute(g_norm_warp_pk<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, 8 * 260 * 4), "norm attribute");
      rc |= cuda_check(cudaFuncSetAttribute(g_norm_warp_pk<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 8 * 516 * 4), "norm attribute");
      rc |= cuda_check(cudaFuncSetAttribute(g_norm_warp_pk<3>, cudaFuncAttributeMaxDynamicSharedMemorySize, 8 * 772 * 4), "norm attribute");
      rc |= cuda_check(cudaFuncSetAttribute(g_norm_warp_pk<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, 8 * 1028 * 4), "norm attribute");
      rc |= cuda_check(cudaFuncSetAttribute(g_norm_warp_pk<5>, cudaFuncAttributeMaxDynamicSharedMemorySize, 8 * 1284 * 4), "norm attribute");
      rc |= cuda_check(cudaFuncSetAttribute(g_norm_warp_pk<6>, cudaFuncAttributeMaxDynamicSharedMemorySize, 8 * 1540 * 4), "norm attribute");
      rc |= cuda_check(cudaFuncSetAttribute(g_norm_warp_pk<7>, cudaFuncAttributeMaxDynamicSharedMemorySize, 8 * 1796 * 4), "norm attribute");
      rc |= cuda_check(cudaFuncSetAttribute(g_norm_warp_pk<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, 8 * 2052 * 4), "norm attribute");
      if (rc) {
        shlo_release(o);
        return 1;
      }
      attr_pk[dev->id] = true;
    }
    int64_t blocks = y_pack[1] / 8;
    if (blocks > (int64_t)dev->sm_count * 8) blocks = (int64_t)dev->sm_count * 8;
    const float *xp = (const float *)data_ptr(x);
    float *yp = (float *)o->buf->ptr;
    const int64_t rp = y_pack[1];
    switch (ncols / 128) {
      case 1: g_norm_warp_pk<1><<<(unsigned)blocks, 256, tbytes, dev->stream>>>(xp, yp, rows, rp, eps, gp, bp); break;
      case 2: g_norm_warp_pk<2><<<(unsigned)blocks, 256, tbytes, dev->stream>>>(xp, yp, rows, rp, eps, gp, bp); break;
      case 3: g_norm_warp_pk<3><<<(unsigned)blocks, 256, tbytes, dev->stream>>>(xp, yp, rows, rp, eps, gp, bp); break;
      case 4: g_norm_warp_pk<4><<<(unsigned)blocks, 256, tbytes, dev->stream>>>(xp, yp, rows, rp, eps, gp, bp); break;
      case 5: g_norm_warp_pk<5><<<(unsigned)blocks, 256, tbytes, dev->stream>>>(xp, yp, rows, rp, eps, gp, bp); break;
      case 6: g_norm_warp_pk<6><<<(unsigned)blocks, 256, tbytes, dev->stream>>>(xp, yp, rows, rp, eps, gp, bp); break;
      case 7: g_norm_warp_pk<7><<<(unsigned)blocks, 256, tbytes, dev->stream>>>(xp, yp, rows, rp, eps, gp, bp); break;
      default: g_norm_warp_pk<8><<<(unsigned)blocks, 256, tbytes, dev->stream>>>(xp, yp, rows, rp, eps, gp, bp); break;
    }
    if (launch_check("norm")) {
      shlo_release(o);
      return 1;
    }
    *out = o;
    return 0;
  }
  if (y_pack) {
    Arr *n, *q;
    SHLO_TRY(k_norm_affine_packed(dev, x, p, gamma, beta, nullptr, &n));
    const int rc = k_pack_x(dev, n, rows, ncols, y_pack, &q);
    shlo_release(n);
    SHLO_TRY(rc);
    *out = q;
    return 0;
  }
  int64_t shape[1] = {ncols * rows};
  Arr *o;
  SHLO_TRY(new_array(dev, kF32, shape, 1, &o));
  if (warp_rows) {
    // one warp a row, the row in registers
    int64_t blocks = (rows + 3) / 4;
    if (blocks > (int64_t)dev->sm_count * 32) blocks = (int64_t)dev->sm_count * 32;
    const float *xp = (const float *)data_ptr(x);
    float *yp = (float *)o->buf->ptr;
    switch (ncols / 128) {
      case 1: g_norm_warp<1><<<(unsigned)blocks, 128, 0, dev->stream>>>(xp, yp, rows, eps, gp, bp); break;
      case 2: g_norm_warp<2><<<(unsigned)blocks, 128, 0, dev->stream>>>(xp, yp, rows, eps, gp, bp); break;
      case 3: g_norm_warp<3><<<(unsigned)blocks, 128, 0, dev->stream>>>(xp, yp, rows, eps, gp, bp); break;
      case 4: g_norm_warp<4><<<(unsigned)blocks, 128, 0, dev->stream>>>(xp, yp, rows, eps, gp, bp); break;
      case 5: g_norm_warp<5><<<(unsigned)blocks, 128, 0, dev->stream>>>(xp, yp, rows, eps, gp, bp); break;
      case 6: g_norm_warp<6><<<(unsigned)blocks, 128, 0, dev->stream>>>(xp, yp, rows, eps, gp, bp); break;
      case 7: g_norm_warp<7><<<(unsigned)blocks, 128, 0, dev->stream>>>(xp, yp, rows, eps, gp, bp); break;
      default: g_norm_warp<8><<<(unsigned)blocks, 128, 0, dev->stream>>>(xp, yp, rows, eps, gp, bp); break;
    }
    if (launch_check("norm")) {
      shlo_release(o);
      return 1;
    }
  } else if (ncols * rows > 0 && p[3] == 0 && ncols % 4 == 0 && ncols <= 1024 && aligned) {
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

// gelu_erf: Shaders.lean:186-199 (gelu.cuh has the arithmetic).
// The planted fault: GELU's tanh form (SQRT_2_OVER_PI, GELU_COEF_A of vec.h).
__device__ __forceinline__ float gelu_tanh_one(float v) {
  const float ev = tanhf(__fmul_rn(__fmul_rn(bitsf(0x3F4C422Au), v),
                                   __fadd_rn(1.0f, __fmul_rn(__fmul_rn(bitsf(0x3D372713u), v), v))));
  return gelu_nan(v, gelu_of(v, ev));
}

// A grid-stride loop over 16-byte vectors, the next vector's load issued before
// the current one is computed; 64 registers a thread, so that four blocks of 256
// threads stay resident on a multiprocessor (a few spills, on the rare path).
__global__ void __launch_bounds__(256, 4) g_gelu_erf(const float *__restrict__ x, float *__restrict__ y, int64_t n, int gpu_erf) {
  __shared__ shlo_erf::ErfSmem tab;
  shlo_erf::erf_smem_load(&tab);
  __syncthreads();
  const shlo_erf::ErfSmem *t = &tab;
  if (gpu_erf) {
    map_f32(x, y, n, [](float v) { return gelu_tanh_one(v); });
    return;
  }
  const int64_t nv = n >> 2;
  const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, stride = (int64_t)gridDim.x * blockDim.x;
  const float4 *xv = reinterpret_cast<const float4 *>(x);
  float4 *yv = reinterpret_cast<float4 *>(y);
  int64_t i = t0;
  if (i < nv) {
    float4 cur = __ldg(xv + i);
    for (; i + stride < nv; i += stride) {
      const float4 nxt = __ldg(xv + i + stride);
      yv[i] = gelu4(cur, t);
      cur = nxt;
    }
    yv[i] = gelu4(cur, t);
  }
  for (int64_t j = 4 * nv + t0; j < n; j += stride) {
    const float v = x[j];
    y[j] = gelu_nan(v, gelu_of(v, shlo_erf::erff_cr_smem(__fmul_rn(v, bitsf(0x3F3504F3u)), t)));
  }
}

// erff_map: Shaders.lean:204-208: y[t] = bits(erff(bits^-1(base + t))), four
// consecutive patterns per thread and trip, stored as one 16-byte vector.
__global__ void __launch_bounds__(256, 4) g_erff_map(uint32_t base, int64_t n, uint32_t *__restrict__ y) {
  __shared__ shlo_erf::ErfSmem tab;
  shlo_erf::erf_smem_load(&tab);
  __syncthreads();
  const shlo_erf::ErfSmem *t = &tab;
  const int64_t nv = n >> 2;
  const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = t0; i < nv; i += stride) {
    const uint32_t p = base + (uint32_t)(4 * i);
    const float x[4] = {bitsf(p), bitsf(p + 1u), bitsf(p + 2u), bitsf(p + 3u)};
    float r[4];
    shlo_erf::erff4_smem(x, r, t);
    reinterpret_cast<uint4 *>(y)[i] = make_uint4(fbits(r[0]), fbits(r[1]), fbits(r[2]), fbits(r[3]));
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

// The erf kernels stage a 16 KB table in every block, so they run one resident
// wave of blocks over a grid-stride loop rather than launch_ew's 16 a
// multiprocessor.
template <typename K, typename... Args>
static int launch_erf(Device *dev, int64_t n, K kernel, std::atomic<int> *per_sm, const char *what, Args... args) {
  if (n <= 0) return 0;
  int b = per_sm->load();
  if (b == 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kernel, 256, 0) != cudaSuccess || b < 1) b = 1;
    per_sm->store(b);
  }
  kernel<<<grid_for(n, 256, dev, b), 256, 0, dev->stream>>>(args...);
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
    return fail("%s", kGeluStockRefusal);
  Arr *o;
  SHLO_TRY(simple_out(dev, kF32, n, &o));
  static std::atomic<int> per_sm{0};
  const int rc = launch_erf(dev, n, g_gelu_erf, &per_sm, "gelu_erf", (const float *)data_ptr(x), (float *)o->buf->ptr,
                            n, (int)(p[1] != 0));
  if (rc) {
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
  static std::atomic<int> per_sm{0};
  const int rc = launch_erf(dev, n, g_erff_map, &per_sm, "erff_map", p[0], n, (uint32_t *)o->buf->ptr);
  if (rc) {
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

// The kernel's dynamic shared-memory limit, raised once per device (with that
// device current).
static bool g_noalloc_attr[64];

static int noalloc_smem_attr(int dev, int smem) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_attr[dev]) {
    cudaError_t e = cudaFuncSetAttribute(k_mul_mat_fast, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return cuda_check(e, "mul_mat_noalloc: shared-memory limit");
    g_noalloc_attr[dev] = true;
  }
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
  MMArgs a{};  // the epilogue fields (bias, residual, park slabs) stay null: this kernel has none
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
  SHLO_TRY(noalloc_smem_attr(devid, (int)smem));
  dim3 grid(Mp / mm::BM, (unsigned)(Bx * a.r_tiles));
  k_mul_mat_fast<<<grid, mm::THREADS, smem, s>>>(a);
  return launch_check("mul_mat_noalloc");
}
