// Built-in ops of the boundary (c/smlx_shim.c:142-264, 405-414): unary and binary
// elementwise ops with numpy broadcasting and MLX type promotion, where, astype,
// concat, take, max along an axis, count_nonzero, the built-in matmul, and the
// strided copies behind contiguous/reshape.
//
// Every op here is one correctly rounded operation per element (or pure data
// movement), so its result does not depend on evaluation order; that is the
// exactness argument of StablehloMlx/Lower.lean:13-17. The two deliberate
// exceptions are the ones the reference's tests require to be inexact
// (Tests/OpTests.lean:120, 259-264): built-in float `/` uses the GPU's
// approximate division, and built-in matmul sums in plain k order.
#include <cmath>
#include <type_traits>

#include "common.cuh"

namespace shlo {

// ------------------------------------------------------------ iteration ----

struct Iter {
  int ndim;
  int64_t n;
  int64_t shape[kMaxRank];
};
struct Operand {
  const char *ptr;
  int dtype;
  int64_t strides[kMaxRank];
};

// Merge adjacent axes that every operand walks contiguously; drop size-1 axes.
static void collapse(Iter &it, Operand *ops, int nops) {
  int64_t shape[kMaxRank];
  int64_t st[8][kMaxRank];
  int nd = 0;
  for (int d = 0; d < it.ndim; d++) {
    if (it.shape[d] == 1) continue;
    if (nd > 0) {
      bool merge = true;
      for (int k = 0; k < nops; k++)
        if (st[k][nd - 1] != ops[k].strides[d] * it.shape[d]) merge = false;
      if (merge) {
        shape[nd - 1] *= it.shape[d];
        for (int k = 0; k < nops; k++) st[k][nd - 1] = ops[k].strides[d];
        continue;
      }
    }
    shape[nd] = it.shape[d];
    for (int k = 0; k < nops; k++) st[k][nd] = ops[k].strides[d];
    nd++;
  }
  it.ndim = nd;
  for (int d = 0; d < nd; d++) {
    it.shape[d] = shape[d];
    for (int k = 0; k < nops; k++) ops[k].strides[d] = st[k][d];
  }
}

// Offsets of element `idx` (row-major over it.shape) in two to four operands.
// ND is the collapsed rank (1, 2, 3) or kMaxRank for any rank; I is the index
// type (32-bit whenever the element count allows). The dimension loops are
// unrolled so every shape/stride access is a fixed parameter-space offset.
template <int ND, typename I>
__device__ __forceinline__ void offs2(const Iter &it, const Operand &a, const Operand &b, I idx, int64_t &oa,
                                      int64_t &ob) {
  oa = 0;
  ob = 0;
#pragma unroll
  for (int d = ND - 1; d >= 0; d--) {
    if (ND == kMaxRank && d >= it.ndim) continue;
    I c = idx;
    if (d > 0) {
      I s = (I)it.shape[d];
      I q = idx / s;
      c = idx - q * s;
      idx = q;
    }
    oa += (int64_t)c * a.strides[d];
    ob += (int64_t)c * b.strides[d];
  }
}

template <int ND, typename I>
__device__ __forceinline__ void offs3(const Iter &it, const Operand &a, const Operand &b, const Operand &z, I idx,
                                      int64_t &oa, int64_t &ob, int64_t &oz) {
  oa = 0;
  ob = 0;
  oz = 0;
#pragma unroll
  for (int d = ND - 1; d >= 0; d--) {
    if (ND == kMaxRank && d >= it.ndim) continue;
    I c = idx;
    if (d > 0) {
      I s = (I)it.shape[d];
      I q = idx / s;
      c = idx - q * s;
      idx = q;
    }
    oa += (int64_t)c * a.strides[d];
    ob += (int64_t)c * b.strides[d];
    oz += (int64_t)c * z.strides[d];
  }
}

template <int ND, typename I>
__device__ __forceinline__ void offs4(const Iter &it, const Operand &a, const Operand &b, const Operand &c3,
                                      const Operand &z, I idx, int64_t &oa, int64_t &ob, int64_t &oc, int64_t &oz) {
  oa = 0;
  ob = 0;
  oc = 0;
  oz = 0;
#pragma unroll
  for (int d = ND - 1; d >= 0; d--) {
    if (ND == kMaxRank && d >= it.ndim) continue;
    I c = idx;
    if (d > 0) {
      I s = (I)it.shape[d];
      I q = idx / s;
      c = idx - q * s;
      idx = q;
    }
    oa += (int64_t)c * a.strides[d];
    ob += (int64_t)c * b.strides[d];
    oc += (int64_t)c * c3.strides[d];
    oz += (int64_t)c * z.strides[d];
  }
}

// Call f(integral_constant<ND>, I{}) with the rank and index type for `it`.
template <typename F>
static void by_rank(const Iter &it, F &&f) {
  if (it.n < ((int64_t)1 << 31)) {
    switch (it.ndim) {
      case 1: f(std::integral_constant<int, 1>{}, uint32_t{}); return;
      case 2: f(std::integral_constant<int, 2>{}, uint32_t{}); return;
      case 3: f(std::integral_constant<int, 3>{}, uint32_t{}); return;
      default: f(std::integral_constant<int, kMaxRank>{}, uint32_t{}); return;
    }
  }
  f(std::integral_constant<int, kMaxRank>{}, uint64_t{});
}

#define GRID_LOOP(I, i, n)                                                                     \
  for (I i = (I)blockIdx.x * blockDim.x + threadIdx.x, _st = (I)gridDim.x * blockDim.x; i < (I)(n); \
       i += _st)

// ------------------------------------------------------------ typed access ----

template <typename T>
__device__ __forceinline__ T load_as(const char *base, int dt, int64_t i) {
  switch (dt) {
    case kBool: return (T)(reinterpret_cast<const uint8_t *>(base)[i] != 0);
    case kU8: return (T)reinterpret_cast<const uint8_t *>(base)[i];
    case kU16: return (T)reinterpret_cast<const uint16_t *>(base)[i];
    case kU32: return (T)reinterpret_cast<const uint32_t *>(base)[i];
    case kU64: return (T)reinterpret_cast<const uint64_t *>(base)[i];
    case kI8: return (T)reinterpret_cast<const int8_t *>(base)[i];
    case kI16: return (T)reinterpret_cast<const int16_t *>(base)[i];
    case kI32: return (T)reinterpret_cast<const int32_t *>(base)[i];
    case kI64: return (T)reinterpret_cast<const int64_t *>(base)[i];
    case kF16: return (T)__half2float(reinterpret_cast<const __half *>(base)[i]);
    default: return (T)reinterpret_cast<const float *>(base)[i];
  }
}

// Float -> integer conversions saturate (NaN -> 0), as the GPU's cvt does.
template <typename T>
__device__ __forceinline__ void store_as(char *base, int dt, int64_t i, T v) {
  switch (dt) {
    case kBool: reinterpret_cast<uint8_t *>(base)[i] = (v != (T)0); break;
    case kU8: reinterpret_cast<uint8_t *>(base)[i] = (uint8_t)v; break;
    case kU16: reinterpret_cast<uint16_t *>(base)[i] = (uint16_t)v; break;
    case kU32: reinterpret_cast<uint32_t *>(base)[i] = (uint32_t)v; break;
    case kU64: reinterpret_cast<uint64_t *>(base)[i] = (uint64_t)v; break;
    case kI8: reinterpret_cast<int8_t *>(base)[i] = (int8_t)v; break;
    case kI16: reinterpret_cast<int16_t *>(base)[i] = (int16_t)v; break;
    case kI32: reinterpret_cast<int32_t *>(base)[i] = (int32_t)v; break;
    case kI64: reinterpret_cast<int64_t *>(base)[i] = (int64_t)v; break;
    case kF16: reinterpret_cast<__half *>(base)[i] = __float2half_rn((float)v); break;
    default: reinterpret_cast<float *>(base)[i] = (float)v; break;
  }
}

// Exact conversions between float and the integer types for astype: float ->
// integer truncates toward zero and saturates, NaN -> 0 (the GPU's cvt.rzi).
template <typename D>
__device__ __forceinline__ D f2i(float v) {
  if (v != v) return (D)0;
  if (sizeof(D) == 8) {
    if (std::is_signed<D>::value) return (D)__float2ll_rz(v);
    return (D)__float2ull_rz(v);
  }
  if (std::is_signed<D>::value) {
    long long t = __float2ll_rz(v);
    long long lo = sizeof(D) == 1 ? -128 : sizeof(D) == 2 ? -32768 : -2147483648LL;
    long long hi = sizeof(D) == 1 ? 127 : sizeof(D) == 2 ? 32767 : 2147483647LL;
    return (D)(t < lo ? lo : t > hi ? hi : t);
  }
  unsigned long long t = v <= 0.0f ? 0ull : __float2ull_rz(v);
  unsigned long long hi = sizeof(D) == 1 ? 255ull : sizeof(D) == 2 ? 65535ull : 4294967295ull;
  return (D)(t > hi ? hi : t);
}

// ------------------------------------------------------------ strided copy ----

template <typename E, int ND, typename I>
__global__ void k_copy(Iter it, Operand src, Operand dst) {
  GRID_LOOP(I, i, it.n) {
    int64_t os, od;
    offs2<ND, I>(it, src, dst, i, os, od);
    reinterpret_cast<E *>(const_cast<char *>(dst.ptr))[od] = reinterpret_cast<const E *>(src.ptr)[os];
  }
}

// Rows that are contiguous in both source and destination, with up to three
// outer axes of any strides; V is the widest vector the alignment allows.
struct RowDesc {
  const void *src;
  void *dst;
  uint32_t nrows, lenv;  // rows, row length in V units
  int no;                // outer axes (0..3)
  uint32_t os[3];        // outer shape
  int64_t ss[3], ds[3];  // outer strides, in V units
};

template <typename V>
__global__ void k_copy_rows(RowDesc d) {
  const uint32_t total = d.nrows * d.lenv;
  GRID_LOOP(uint32_t, i, total) {
    uint32_t r = i / d.lenv, c = i - r * d.lenv;
    int64_t so = 0, dof = 0;
#pragma unroll
    for (int k = 2; k >= 0; k--) {
      if (k >= d.no) continue;
      uint32_t cc = r;
      if (k > 0) {
        uint32_t q = r / d.os[k];
        cc = r - q * d.os[k];
        r = q;
      }
      so += (int64_t)cc * d.ss[k];
      dof += (int64_t)cc * d.ds[k];
    }
    reinterpret_cast<V *>(d.dst)[dof + c] = reinterpret_cast<const V *>(d.src)[so + c];
  }
}

// A transposing copy: the source is contiguous along axis t, the destination
// along the last axis l. 32x32 tiles through shared memory keep both sides
// coalesced; up to three outer axes run over blockIdx.z.
struct TDesc {
  const char *src;
  char *dst;
  int64_t n_t, n_l;
  int64_t ss_l, ds_t;    // source stride of l, destination stride of t (elements)
  int no;
  uint32_t nouter;
  uint32_t os[3];
  int64_t ss[3], ds[3];
};

template <typename E>
__global__ void k_copy_transpose(TDesc d) {
  __shared__ E tile[32][33];
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int64_t t0 = (int64_t)blockIdx.y * 32, l0 = (int64_t)blockIdx.x * 32;
  for (uint32_t z = blockIdx.z; z < d.nouter; z += gridDim.z) {
    int64_t so = 0, dof = 0;
    uint32_t r = z;
#pragma unroll
    for (int k = 2; k >= 0; k--) {
      if (k >= d.no) continue;
      uint32_t cc = r;
      if (k > 0) {
        uint32_t q = r / d.os[k];
        cc = r - q * d.os[k];
        r = q;
      }
      so += (int64_t)cc * d.ss[k];
      dof += (int64_t)cc * d.ds[k];
    }
    const E *src = reinterpret_cast<const E *>(d.src) + so;
    E *dst = reinterpret_cast<E *>(d.dst) + dof;
#pragma unroll
    for (int j = 0; j < 32; j += 8) {
      int64_t t = t0 + tx, l = l0 + ty + j;
      if (t < d.n_t && l < d.n_l) tile[ty + j][tx] = src[t + l * d.ss_l];
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < 32; j += 8) {
      int64_t t = t0 + ty + j, l = l0 + tx;
      if (t < d.n_t && l < d.n_l) dst[t * d.ds_t + l] = tile[tx][ty + j];
    }
    __syncthreads();
  }
}

template <typename E>
static void launch_transpose(Device *dev, const TDesc &d) {
  dim3 grid((unsigned)((d.n_l + 31) / 32), (unsigned)((d.n_t + 31) / 32), d.nouter < 65535 ? d.nouter : 65535);
  k_copy_transpose<E><<<grid, dim3(32, 8), 0, dev->stream>>>(d);
}

static bool aligned(const void *p, size_t a) { return ((uintptr_t)p % a) == 0; }

// Copy the strided `src` into `dst` laid out with strides `dst_strides`.
static int copy_into(Device *dev, const Arr *src, char *dst, const int64_t *dst_strides) {
  Iter it;
  it.ndim = src->ndim;
  it.n = numel(src);
  if (it.n == 0) return 0;
  for (int d = 0; d < src->ndim; d++) it.shape[d] = src->shape[d];
  Operand ops[2];
  ops[0].ptr = data_ptr(src);
  ops[0].dtype = src->dtype;
  ops[1].ptr = dst;
  ops[1].dtype = src->dtype;
  for (int d = 0; d < src->ndim; d++) {
    ops[0].strides[d] = src->strides[d];
    ops[1].strides[d] = dst_strides[d];
  }
  collapse(it, ops, 2);
  if (it.ndim == 0) {
    it.ndim = 1;
    it.shape[0] = 1;
    ops[0].strides[0] = ops[1].strides[0] = 1;
  }
  const size_t es = dtype_size(src->dtype);
  const int nd = it.ndim, last = nd - 1;
  // Fast path 1: rows contiguous on both sides.
  if (nd <= 4 && ops[0].strides[last] == 1 && ops[1].strides[last] == 1 && it.n < ((int64_t)1 << 31)) {
    int64_t len = it.shape[last];
    size_t vb = es;  // vector bytes
    for (size_t cand = 16; cand > es; cand /= 2) {
      int64_t k = (int64_t)(cand / es);
      bool ok = len % k == 0 && aligned(ops[0].ptr, cand) && aligned(ops[1].ptr, cand);
      for (int d = 0; d < last && ok; d++) ok = ops[0].strides[d] % k == 0 && ops[1].strides[d] % k == 0;
      if (ok) {
        vb = cand;
        break;
      }
    }
    const int64_t k = (int64_t)(vb / es);
    RowDesc d;
    d.src = ops[0].ptr;
    d.dst = (void *)ops[1].ptr;
    d.lenv = (uint32_t)(len / k);
    d.nrows = (uint32_t)(it.n / len);
    d.no = last;
    for (int a = 0; a < last; a++) {
      d.os[a] = (uint32_t)it.shape[a];
      d.ss[a] = ops[0].strides[a] / k;
      d.ds[a] = ops[1].strides[a] / k;
    }
    unsigned g = grid_for((int64_t)d.nrows * d.lenv, 256, dev, 16);
    switch (vb) {
      case 16: k_copy_rows<uint4><<<g, 256, 0, dev->stream>>>(d); break;
      case 8: k_copy_rows<uint2><<<g, 256, 0, dev->stream>>>(d); break;
      case 4: k_copy_rows<uint32_t><<<g, 256, 0, dev->stream>>>(d); break;
      case 2: k_copy_rows<uint16_t><<<g, 256, 0, dev->stream>>>(d); break;
      default: k_copy_rows<uint8_t><<<g, 256, 0, dev->stream>>>(d); break;
    }
    return launch_check("copy");
  }
  // Fast path 2: a transpose (source contiguous along another axis than the last).
  if (nd >= 2 && nd <= 5 && ops[1].strides[last] == 1 && ops[0].strides[last] != 1) {
    int t = -1;
    for (int a = 0; a < last; a++)
      if (ops[0].strides[a] == 1) t = a;
    int64_t nouter = it.n / (it.shape[t < 0 ? 0 : t] * it.shape[last]);
    if (t >= 0 && nouter < ((int64_t)1 << 31) && it.shape[t] < 65535 * 32) {
      TDesc d;
      d.src = ops[0].ptr;
      d.dst = (char *)ops[1].ptr;
      d.n_t = it.shape[t];
      d.n_l = it.shape[last];
      d.ss_l = ops[0].strides[last];
      d.ds_t = ops[1].strides[t];
      d.no = 0;
      for (int a = 0; a < last; a++) {
        if (a == t) continue;
        d.os[d.no] = (uint32_t)it.shape[a];
        d.ss[d.no] = ops[0].strides[a];
        d.ds[d.no] = ops[1].strides[a];
        d.no++;
      }
      d.nouter = (uint32_t)nouter;
      switch (es) {
        case 1: launch_transpose<uint8_t>(dev, d); break;
        case 2: launch_transpose<uint16_t>(dev, d); break;
        case 4: launch_transpose<uint32_t>(dev, d); break;
        default: launch_transpose<uint64_t>(dev, d); break;
      }
      return launch_check("copy (transpose)");
    }
  }
  unsigned g = grid_for(it.n, 256, dev, 16);
  by_rank(it, [&](auto ndc, auto ic) {
    constexpr int ND = decltype(ndc)::value;
    using I = decltype(ic);
    switch (es) {
      case 1: k_copy<uint8_t, ND, I><<<g, 256, 0, dev->stream>>>(it, ops[0], ops[1]); break;
      case 2: k_copy<uint16_t, ND, I><<<g, 256, 0, dev->stream>>>(it, ops[0], ops[1]); break;
      case 4: k_copy<uint32_t, ND, I><<<g, 256, 0, dev->stream>>>(it, ops[0], ops[1]); break;
      default: k_copy<uint64_t, ND, I><<<g, 256, 0, dev->stream>>>(it, ops[0], ops[1]); break;
    }
  });
  return launch_check("copy");
}

int launch_copy_strided(Device *dev, const Arr *src, void *dst) {
  Arr tmp;
  tmp.ndim = src->ndim;
  for (int d = 0; d < src->ndim; d++) tmp.shape[d] = src->shape[d];
  set_row_major(&tmp);
  return copy_into(dev, src, static_cast<char *>(dst), tmp.strides);
}

// ------------------------------------------------------------ astype ----

template <typename C, int ND, typename I>
__global__ void k_cast(Iter it, Operand src, Operand dst) {
  GRID_LOOP(I, i, it.n) {
    int64_t os, od;
    offs2<ND, I>(it, src, dst, i, os, od);
    C v = load_as<C>(src.ptr, src.dtype, os);
    store_as<C>(const_cast<char *>(dst.ptr), dst.dtype, od, v);
  }
}

// float -> integer with saturation
template <typename D, int ND, typename I>
__global__ void k_cast_f2i(Iter it, Operand src, Operand dst) {
  GRID_LOOP(I, i, it.n) {
    int64_t os, od;
    offs2<ND, I>(it, src, dst, i, os, od);
    float v = load_as<float>(src.ptr, src.dtype, os);
    reinterpret_cast<D *>(const_cast<char *>(dst.ptr))[od] = f2i<D>(v);
  }
}

template <typename K, typename... Args>
static void launch_typed(K kernel, unsigned g, Device *dev, Args... args) {
  kernel<<<g, 256, 0, dev->stream>>>(args...);
}

int cast_array(Arr *a, uint8_t dt, Arr **out) {
  if (!dtype_valid(dt)) return fail("astype: dtype %d not carried", (int)dt);
  if (a->dtype == dt) {
    a->rc.fetch_add(1);
    *out = a;
    return 0;
  }
  Device *dev;
  SHLO_TRY(arr_device(a, &dev));
  Arr *o;
  SHLO_TRY(new_array(dev, dt, a->shape, a->ndim, &o));
  Iter it;
  it.ndim = a->ndim;
  it.n = numel(a);
  for (int d = 0; d < a->ndim; d++) it.shape[d] = a->shape[d];
  Operand ops[2];
  ops[0].ptr = data_ptr(a);
  ops[0].dtype = a->dtype;
  ops[1].ptr = (const char *)o->buf->ptr;
  ops[1].dtype = dt;
  for (int d = 0; d < a->ndim; d++) {
    ops[0].strides[d] = a->strides[d];
    ops[1].strides[d] = o->strides[d];
  }
  collapse(it, ops, 2);
  if (it.ndim == 0) {
    it.ndim = 1;
    it.shape[0] = 1;
    ops[0].strides[0] = ops[1].strides[0] = 1;
  }
  if (it.n > 0) {
    unsigned g = grid_for(it.n, 256, dev, 16);
    bool from_float = dtype_is_float(a->dtype);
    by_rank(it, [&](auto ndc, auto ic) {
      constexpr int ND = decltype(ndc)::value;
      using I = decltype(ic);
      if (from_float && !dtype_is_float(dt) && dt != kBool) {
        switch (dt) {
          case kU8: launch_typed(k_cast_f2i<uint8_t, ND, I>, g, dev, it, ops[0], ops[1]); break;
          case kU16: launch_typed(k_cast_f2i<uint16_t, ND, I>, g, dev, it, ops[0], ops[1]); break;
          case kU32: launch_typed(k_cast_f2i<uint32_t, ND, I>, g, dev, it, ops[0], ops[1]); break;
          case kU64: launch_typed(k_cast_f2i<uint64_t, ND, I>, g, dev, it, ops[0], ops[1]); break;
          case kI8: launch_typed(k_cast_f2i<int8_t, ND, I>, g, dev, it, ops[0], ops[1]); break;
          case kI16: launch_typed(k_cast_f2i<int16_t, ND, I>, g, dev, it, ops[0], ops[1]); break;
          case kI32: launch_typed(k_cast_f2i<int32_t, ND, I>, g, dev, it, ops[0], ops[1]); break;
          default: launch_typed(k_cast_f2i<int64_t, ND, I>, g, dev, it, ops[0], ops[1]); break;
        }
      } else if (from_float || dtype_is_float(dt)) {
        // int -> float rounds once (int64/uint64 sources go through double,
        // which is exact up to 2^53 and rounds once to binary32 beyond that for
        // all but a vanishing set of ties).
        if (a->dtype == kI64 || a->dtype == kU64)
          launch_typed(k_cast<double, ND, I>, g, dev, it, ops[0], ops[1]);
        else
          launch_typed(k_cast<float, ND, I>, g, dev, it, ops[0], ops[1]);
      } else if (dtype_is_signed_int(a->dtype) || a->dtype == kBool) {
        launch_typed(k_cast<int64_t, ND, I>, g, dev, it, ops[0], ops[1]);
      } else {
        launch_typed(k_cast<uint64_t, ND, I>, g, dev, it, ops[0], ops[1]);
      }
    });
    if (launch_check("astype")) {
      shlo_release(o);
      return 1;
    }
  }
  *out = o;
  return 0;
}

int op_astype(Arr *a, uint8_t dt, Arr **out) { return cast_array(a, dt, out); }

// ------------------------------------------------------------ unary ----

enum { U_NEG, U_ABS, U_SQRT, U_FLOOR, U_EXP, U_ERF, U_NOT, U_INVERT, U_RSQRT, U_TANH, U_SIGMOID };

template <typename C>
__device__ __forceinline__ C unary_int(int op, C v) {
  switch (op) {
    case U_NEG: return (C)(0 - v);
    case U_ABS: return std::is_signed<C>::value ? (v < (C)0 ? (C)(0 - v) : v) : v;
    case U_NOT: return (C)(v == (C)0);
    case U_INVERT: return (C)~v;
    default: return v;  // floor
  }
}

__device__ __forceinline__ float unary_float(int op, float v) {
  switch (op) {
    case U_NEG: return -v;
    case U_ABS: return fabsf(v);
    case U_SQRT: return __fsqrt_rn(v);
    case U_FLOOR: return floorf(v);
    case U_EXP: return expf(v);
    case U_ERF: return erff(v);
    case U_NOT: return (float)(v == 0.0f);
    case U_RSQRT: return rsqrtf(v);
    case U_TANH: return tanhf(v);
    default: return 1.0f / (1.0f + expf(-v));  // sigmoid
  }
}

template <typename C, bool FLOAT, int ND, typename I>
__global__ void k_unary(int op, Iter it, Operand x, Operand y) {
  GRID_LOOP(I, i, it.n) {
    int64_t ox, oy;
    offs2<ND, I>(it, x, y, i, ox, oy);
    if constexpr (FLOAT) {
      float v = load_as<float>(x.ptr, x.dtype, ox);
      store_as<float>(const_cast<char *>(y.ptr), y.dtype, oy, unary_float(op, v));
    } else {
      C v = load_as<C>(x.ptr, x.dtype, ox);
      store_as<C>(const_cast<char *>(y.ptr), y.dtype, oy, unary_int<C>(op, v));
    }
  }
}

// Run an elementwise kernel over `outs` (row-major) and inputs given as views
// already broadcast to the output shape.
static int prepare_iter(Arr *o, Arr *const *ins, int nin, Iter &it, Operand *ops) {
  it.ndim = o->ndim;
  it.n = numel(o);
  for (int d = 0; d < o->ndim; d++) it.shape[d] = o->shape[d];
  for (int k = 0; k < nin; k++) {
    ops[k].ptr = data_ptr(ins[k]);
    ops[k].dtype = ins[k]->dtype;
    for (int d = 0; d < o->ndim; d++) ops[k].strides[d] = ins[k]->strides[d];
  }
  ops[nin].ptr = (const char *)o->buf->ptr;
  ops[nin].dtype = o->dtype;
  for (int d = 0; d < o->ndim; d++) ops[nin].strides[d] = o->strides[d];
  collapse(it, ops, nin + 1);
  if (it.ndim == 0) {
    it.ndim = 1;
    it.shape[0] = 1;
    for (int k = 0; k <= nin; k++) ops[k].strides[0] = 1;
  }
  return 0;
}

int op_unary(uint32_t op, Arr *a, Arr **out) {
  if (op > U_SIGMOID) return fail("unary: unknown op code %u", op);
  Device *dev;
  SHLO_TRY(arr_device(a, &dev));
  int dt = a->dtype;
  bool needs_float = op == U_SQRT || op == U_EXP || op == U_ERF || op == U_RSQRT || op == U_TANH || op == U_SIGMOID;
  int odt = dt;
  if (needs_float && !dtype_is_float(dt)) odt = kF32;
  if (op == U_NOT) odt = kBool;
  if (op == U_NEG && dt == kBool) return fail("unary: negative of bool not carried");
  if (op == U_INVERT && dtype_is_float(dt)) return fail("unary: bitwise_invert of %s not carried", dtype_name(dt));
  Arr *o;
  SHLO_TRY(new_array(dev, (uint8_t)odt, a->shape, a->ndim, &o));
  Iter it;
  Operand ops[2];
  prepare_iter(o, &a, 1, it, ops);
  if (it.n > 0) {
    unsigned g = grid_for(it.n, 256, dev, 16);
    bool flt = dtype_is_float(dt) || needs_float;
    int uop = (dt == kBool && op == U_INVERT) ? (int)U_NOT : (int)op;  // bool: invert is logical not
    by_rank(it, [&](auto ndc, auto ic) {
      constexpr int ND = decltype(ndc)::value;
      using I = decltype(ic);
      if (flt) {
        launch_typed(k_unary<float, true, ND, I>, g, dev, uop, it, ops[0], ops[1]);
        return;
      }
      switch (dt) {
        case kBool:
        case kU8: launch_typed(k_unary<uint8_t, false, ND, I>, g, dev, uop, it, ops[0], ops[1]); break;
        case kU16: launch_typed(k_unary<uint16_t, false, ND, I>, g, dev, uop, it, ops[0], ops[1]); break;
        case kU32: launch_typed(k_unary<uint32_t, false, ND, I>, g, dev, uop, it, ops[0], ops[1]); break;
        case kU64: launch_typed(k_unary<uint64_t, false, ND, I>, g, dev, uop, it, ops[0], ops[1]); break;
        case kI8: launch_typed(k_unary<int8_t, false, ND, I>, g, dev, uop, it, ops[0], ops[1]); break;
        case kI16: launch_typed(k_unary<int16_t, false, ND, I>, g, dev, uop, it, ops[0], ops[1]); break;
        case kI32: launch_typed(k_unary<int32_t, false, ND, I>, g, dev, uop, it, ops[0], ops[1]); break;
        default: launch_typed(k_unary<int64_t, false, ND, I>, g, dev, uop, it, ops[0], ops[1]); break;
      }
    });
    if (launch_check("unary")) {
      shlo_release(o);
      return 1;
    }
  }
  *out = o;
  return 0;
}

// ------------------------------------------------------------ binary ----

enum {
  B_ADD, B_SUB, B_MUL, B_DIV, B_MAX, B_MIN, B_AND, B_OR, B_XOR, B_SHL, B_SHR, B_EQ, B_NE, B_LT, B_LE,
  B_GT, B_GE, B_MATMUL, B_REM, B_LAND, B_LOR
};

static bool is_compare(int op) { return op >= B_EQ && op <= B_GE; }

template <typename C>
__device__ __forceinline__ bool compare(int op, C u, C v) {
  switch (op) {
    case B_EQ: return u == v;
    case B_NE: return u != v;
    case B_LT: return u < v;
    case B_LE: return u <= v;
    case B_GT: return u > v;
    default: return u >= v;
  }
}

template <typename C>
__device__ __forceinline__ C binary_int(int op, C u, C v) {
  const int bits = (int)sizeof(C) * 8;
  switch (op) {
    case B_ADD: return (C)(u + v);
    case B_SUB: return (C)(u - v);
    case B_MUL: return (C)(u * v);
    case B_DIV: return v == (C)0 ? (C)0 : (C)(u / v);
    case B_MAX: return u > v ? u : v;
    case B_MIN: return u < v ? u : v;
    case B_AND: return (C)(u & v);
    case B_OR: return (C)(u | v);
    case B_XOR: return (C)(u ^ v);
    case B_SHL: return ((uint64_t)v >= (uint64_t)bits) ? (C)0 : (C)(u << v);
    case B_SHR:
      if ((uint64_t)v >= (uint64_t)bits) return (std::is_signed<C>::value && u < (C)0) ? (C)-1 : (C)0;
      return (C)(u >> v);
    case B_REM: {
      if (v == (C)0) return (C)0;
      C r = (C)(u % v);
      if (std::is_signed<C>::value && r != (C)0 && ((r < (C)0) != (v < (C)0))) r = (C)(r + v);
      return r;
    }
    case B_LAND: return (C)((u != (C)0) && (v != (C)0));
    default: return (C)((u != (C)0) || (v != (C)0));  // B_LOR
  }
}

__device__ __forceinline__ float binary_float(int op, float u, float v) {
  switch (op) {
    case B_ADD: return __fadd_rn(u, v);
    case B_SUB: return __fsub_rn(u, v);
    case B_MUL: return __fmul_rn(u, v);
    case B_DIV: return __fdividef(u, v);  // the GPU's own (approximate) division
    case B_MAX: return (u != u) ? u : (u > v ? u : v);
    case B_MIN: return (u != u) ? u : (u < v ? u : v);
    case B_REM: {
      float r = fmodf(u, v);
      if (r != 0.0f && ((r < 0.0f) != (v < 0.0f))) r = __fadd_rn(r, v);
      return r;
    }
    case B_LAND: return (float)((u != 0.0f) && (v != 0.0f));
    default: return (float)((u != 0.0f) || (v != 0.0f));  // B_LOR
  }
}

template <typename C, bool FLOAT, int ND, typename I>
__global__ void k_binary(int op, Iter it, Operand x, Operand y, Operand z) {
  const bool cmp = op >= B_EQ && op <= B_GE;
  GRID_LOOP(I, i, it.n) {
    int64_t ox, oy, oz;
    offs3<ND, I>(it, x, y, z, i, ox, oy, oz);
    typedef typename std::conditional<FLOAT, float, C>::type V;
    V u = load_as<V>(x.ptr, x.dtype, ox);
    V v = load_as<V>(y.ptr, y.dtype, oy);
    char *zp = const_cast<char *>(z.ptr);
    if (cmp) {
      reinterpret_cast<uint8_t *>(zp)[oz] = compare<V>(op, u, v) ? 1 : 0;
    } else if constexpr (FLOAT) {
      store_as<float>(zp, z.dtype, oz, binary_float(op, (float)u, (float)v));
    } else {
      store_as<C>(zp, z.dtype, oz, binary_int<C>(op, (C)u, (C)v));
    }
  }
}

// binary32 operands and result laid out as [planes, rows, cols] with
// cols % 4 == 0: each operand walks its columns contiguously (a row segment,
// stride 1) or not at all (one value per row, stride 0), and rows and planes at
// any stride. Four elements per thread with 16-byte accesses: the layout of
// bias adds, norm affines, residual adds and per-sample broadcasts
// ([B, S, D] + [B, 1, D]).
struct VecOperand {
  const float *p;
  int64_t plane;  // plane stride, floats
  int64_t row;    // row stride, floats
  int col;        // 1 = contiguous columns, 0 = one value per row
};

__global__ void k_binary_f32v(int op, uint32_t nv, uint32_t colsv, uint32_t rows, VecOperand a, VecOperand b,
                              float4 *__restrict__ y) {
  GRID_LOOP(uint32_t, v, nv) {
    const uint32_t r = v / colsv, c = (v - r * colsv) * 4;
    const uint32_t pl = r / rows, rr = r - pl * rows;
    const float *ap = a.p + pl * a.plane + rr * a.row, *bp = b.p + pl * b.plane + rr * b.row;
    float4 u, w;
    if (a.col) u = *reinterpret_cast<const float4 *>(ap + c);
    else u.x = u.y = u.z = u.w = *ap;
    if (b.col) w = *reinterpret_cast<const float4 *>(bp + c);
    else w.x = w.y = w.z = w.w = *bp;
    float4 o;
    o.x = binary_float(op, u.x, w.x);
    o.y = binary_float(op, u.y, w.y);
    o.z = binary_float(op, u.z, w.z);
    o.w = binary_float(op, u.w, w.w);
    y[v] = o;
  }
}

// The vectorized layout of `it`'s operands, when it applies (at most three
// axes after collapsing; `rows` counts the rows of one plane).
static bool vec_layout(const Iter &it, const Operand *ops, int nin, uint32_t &planes, uint32_t &rows, uint32_t &cols,
                       VecOperand *vo) {
  if (it.ndim < 1 || it.ndim > 3 || it.n >= ((int64_t)1 << 31)) return false;
  const int last = it.ndim - 1;
  const int64_t C = it.shape[last];
  const int64_t R = it.ndim >= 2 ? it.shape[last - 1] : 1;
  if (C % 4) return false;
  for (int k = 0; k <= nin; k++) {
    if (ops[k].dtype != kF32) return false;
    const int64_t cs = ops[k].strides[last];
    const int64_t rs = it.ndim >= 2 ? ops[k].strides[last - 1] : 0;
    const int64_t ps = it.ndim == 3 ? ops[k].strides[0] : 0;
    if (k == nin) {  // the output: row-major
      if (cs != 1 || (it.ndim >= 2 && rs != C) || (it.ndim == 3 && ps != R * C)) return false;
      if (!aligned(ops[k].ptr, 16)) return false;
      continue;
    }
    if (cs == 1) {
      if (rs % 4 || ps % 4 || !aligned(ops[k].ptr, 16)) return false;
    } else if (cs != 0) {
      return false;
    }
    vo[k].p = reinterpret_cast<const float *>(ops[k].ptr);
    vo[k].plane = ps;
    vo[k].row = rs;
    vo[k].col = cs == 1;
  }
  rows = (uint32_t)R;
  planes = (uint32_t)(it.n / (R * C));
  cols = (uint32_t)C;
  return true;
}

static int builtin_matmul(Arr *a, Arr *b, Arr **out);

int op_binary(uint32_t op, Arr *a, Arr *b, Arr **out) {
  if (op > B_LOR) return fail("binary: unknown op code %u", op);
  if (op == B_MATMUL) return builtin_matmul(a, b, out);
  Device *dev, *dev2;
  SHLO_TRY(arr_device(a, &dev));
  SHLO_TRY(arr_device(b, &dev2));
  if (dev != dev2) return fail("binary: operands on devices %d and %d", dev->id, dev2->id);
  int ct = promote_types(a->dtype, b->dtype);
  if (op == B_DIV && !dtype_is_float(ct)) ct = kF32;  // MLX divide is at least float
  if (op == B_LAND || op == B_LOR) ct = kBool;
  bool bitwise = op == B_AND || op == B_OR || op == B_XOR || op == B_SHL || op == B_SHR;
  if (bitwise && dtype_is_float(ct)) return fail("binary: bitwise op on %s not carried", dtype_name(ct));
  int odt = is_compare(op) ? kBool : ct;
  int64_t shape[kMaxRank];
  int nd;
  SHLO_TRY(broadcast_shapes(a->shape, a->ndim, b->shape, b->ndim, shape, &nd));
  Arr *va, *vb;
  SHLO_TRY(broadcast_view(a, shape, nd, &va));
  if (broadcast_view(b, shape, nd, &vb)) {
    shlo_release(va);
    return 1;
  }
  Arr *o;
  int rc = new_array(dev, (uint8_t)odt, shape, nd, &o);
  if (!rc) {
    Iter it;
    Operand ops[3];
    Arr *ins[2] = {va, vb};
    prepare_iter(o, ins, 2, it, ops);
    if (it.n > 0) {
      unsigned g = grid_for(it.n, 256, dev, 16);
      uint32_t vp, vr, vc;
      VecOperand vo[2];
      if (!is_compare(op) && vec_layout(it, ops, 2, vp, vr, vc, vo)) {
        uint32_t nv = vp * vr * (vc / 4);
        k_binary_f32v<<<grid_for(nv, 256, dev, 16), 256, 0, dev->stream>>>((int)op, nv, vc / 4, vr, vo[0], vo[1],
                                                                          (float4 *)ops[2].ptr);
      } else {
        by_rank(it, [&](auto ndc, auto ic) {
          constexpr int ND = decltype(ndc)::value;
          using I = decltype(ic);
          if (dtype_is_float(ct)) {
            launch_typed(k_binary<float, true, ND, I>, g, dev, (int)op, it, ops[0], ops[1], ops[2]);
            return;
          }
          // bool logical ops are computed on 0/1 in uint8
          switch (ct) {
            case kBool:
            case kU8: launch_typed(k_binary<uint8_t, false, ND, I>, g, dev, (int)op, it, ops[0], ops[1], ops[2]); break;
            case kU16: launch_typed(k_binary<uint16_t, false, ND, I>, g, dev, (int)op, it, ops[0], ops[1], ops[2]); break;
            case kU32: launch_typed(k_binary<uint32_t, false, ND, I>, g, dev, (int)op, it, ops[0], ops[1], ops[2]); break;
            case kU64: launch_typed(k_binary<uint64_t, false, ND, I>, g, dev, (int)op, it, ops[0], ops[1], ops[2]); break;
            case kI8: launch_typed(k_binary<int8_t, false, ND, I>, g, dev, (int)op, it, ops[0], ops[1], ops[2]); break;
            case kI16: launch_typed(k_binary<int16_t, false, ND, I>, g, dev, (int)op, it, ops[0], ops[1], ops[2]); break;
            case kI32: launch_typed(k_binary<int32_t, false, ND, I>, g, dev, (int)op, it, ops[0], ops[1], ops[2]); break;
            default: launch_typed(k_binary<int64_t, false, ND, I>, g, dev, (int)op, it, ops[0], ops[1], ops[2]); break;
          }
        });
      }
      rc = launch_check("binary");
      if (rc) shlo_release(o);
    }
  }
  shlo_release(va);
  shlo_release(vb);
  if (!rc) *out = o;
  return rc;
}

// ------------------------------------------------------------ where ----

template <typename C, int ND, typename I>
__global__ void k_where(Iter it, Operand c, Operand x, Operand y, Operand z) {
  GRID_LOOP(I, i, it.n) {
    int64_t oc, ox, oy, oz;
    offs4<ND, I>(it, c, x, y, z, i, oc, ox, oy, oz);
    bool s = load_as<uint8_t>(c.ptr, c.dtype, oc) != 0;
    C v = s ? load_as<C>(x.ptr, x.dtype, ox) : load_as<C>(y.ptr, y.dtype, oy);
    store_as<C>(const_cast<char *>(z.ptr), z.dtype, oz, v);
  }
}

int op_where(Arr *c, Arr *a, Arr *b, Arr **out) {
  Device *dev;
  SHLO_TRY(arr_device(a, &dev));
  int ct = promote_types(a->dtype, b->dtype);
  int64_t s1[kMaxRank], s2[kMaxRank];
  int n1, n2;
  SHLO_TRY(broadcast_shapes(a->shape, a->ndim, b->shape, b->ndim, s1, &n1));
  SHLO_TRY(broadcast_shapes(c->shape, c->ndim, s1, n1, s2, &n2));
  Arr *vc = nullptr, *va = nullptr, *vb = nullptr, *o = nullptr;
  int rc = broadcast_view(c, s2, n2, &vc) || broadcast_view(a, s2, n2, &va) || broadcast_view(b, s2, n2, &vb) ||
           new_array(dev, (uint8_t)ct, s2, n2, &o);
  if (!rc) {
    Iter it;
    Operand ops[4];
    Arr *ins[3] = {vc, va, vb};
    it.ndim = o->ndim;
    it.n = numel(o);
    for (int d = 0; d < o->ndim; d++) it.shape[d] = o->shape[d];
    for (int k = 0; k < 3; k++) {
      ops[k].ptr = data_ptr(ins[k]);
      ops[k].dtype = ins[k]->dtype;
      for (int d = 0; d < o->ndim; d++) ops[k].strides[d] = ins[k]->strides[d];
    }
    ops[3].ptr = (const char *)o->buf->ptr;
    ops[3].dtype = o->dtype;
    for (int d = 0; d < o->ndim; d++) ops[3].strides[d] = o->strides[d];
    collapse(it, ops, 4);
    if (it.ndim == 0) {
      it.ndim = 1;
      it.shape[0] = 1;
      for (int k = 0; k < 4; k++) ops[k].strides[0] = 1;
    }
    if (it.n > 0) {
      unsigned g = grid_for(it.n, 256, dev, 16);
      by_rank(it, [&](auto ndc, auto ic) {
        constexpr int ND = decltype(ndc)::value;
        using I = decltype(ic);
        if (dtype_is_float(ct)) launch_typed(k_where<float, ND, I>, g, dev, it, ops[0], ops[1], ops[2], ops[3]);
        else if (dtype_is_signed_int(ct)) launch_typed(k_where<int64_t, ND, I>, g, dev, it, ops[0], ops[1], ops[2], ops[3]);
        else launch_typed(k_where<uint64_t, ND, I>, g, dev, it, ops[0], ops[1], ops[2], ops[3]);
      });
      rc = launch_check("where");
    }
  }
  if (vc) shlo_release(vc);
  if (va) shlo_release(va);
  if (vb) shlo_release(vb);
  if (rc) {
    if (o) shlo_release(o);
    return 1;
  }
  *out = o;
  return 0;
}

// ------------------------------------------------------------ max along an axis ----

template <typename C>
__global__ void k_max_axis(int64_t outer, int64_t len, int64_t inner, Operand x, Operand y) {
  int64_t n = outer * inner;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    int64_t o = i / inner, in = i % inner;
    int64_t base = o * len * inner + in;
    C m = load_as<C>(x.ptr, x.dtype, base);
    for (int64_t k = 1; k < len; k++) {
      C v = load_as<C>(x.ptr, x.dtype, base + k * inner);
      if (m != m) break;          // NaN propagates
      if (v != v || v > m) m = v;
    }
    store_as<C>(const_cast<char *>(y.ptr), y.dtype, i, m);
  }
}

int op_max_axis(Arr *a, int axis, Arr **out) {
  if (axis < 0 || axis >= a->ndim) return fail("max_axis: axis %d of a rank-%d array", axis, a->ndim);
  if (a->shape[axis] == 0) return fail("max_axis: empty axis");
  Device *dev;
  SHLO_TRY(arr_device(a, &dev));
  Arr *c;
  SHLO_TRY(make_contiguous(a, &c));
  int64_t outer = 1, inner = 1;
  for (int d = 0; d < axis; d++) outer *= a->shape[d];
  for (int d = axis + 1; d < a->ndim; d++) inner *= a->shape[d];
  int64_t shape[kMaxRank];
  int nd = 0;
  for (int d = 0; d < a->ndim; d++)
    if (d != axis) shape[nd++] = a->shape[d];
  Arr *o;
  int rc = new_array(dev, a->dtype, shape, nd, &o);
  if (!rc && outer * inner > 0) {
    Operand x{data_ptr(c), c->dtype, {0}}, y{(const char *)o->buf->ptr, o->dtype, {0}};
    unsigned g = grid_for(outer * inner, 256, dev);
    int dt = a->dtype;
    if (dtype_is_float(dt)) launch_typed(k_max_axis<float>, g, dev, outer, a->shape[axis], inner, x, y);
    else if (dtype_is_signed_int(dt)) launch_typed(k_max_axis<int64_t>, g, dev, outer, a->shape[axis], inner, x, y);
    else launch_typed(k_max_axis<uint64_t>, g, dev, outer, a->shape[axis], inner, x, y);
    rc = launch_check("max_axis");
    if (rc) shlo_release(o);
  }
  shlo_release(c);
  if (!rc) *out = o;
  return rc;
}

// ------------------------------------------------------------ count_nonzero ----

__global__ void k_count_nonzero(const char *p, int dt, int64_t n, unsigned long long *count) {
  unsigned long long local = 0;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    bool nz;
    switch (dt) {
      case kF32: {
        float v = reinterpret_cast<const float *>(p)[i];
        nz = v != 0.0f;  // NaN counts as nonzero
        break;
      }
      case kF16: nz = __half2float(reinterpret_cast<const __half *>(p)[i]) != 0.0f; break;
      default: {
        size_t s = dt == kU64 || dt == kI64 ? 8 : dt == kU32 || dt == kI32 ? 4 : dt == kU16 || dt == kI16 ? 2 : 1;
        uint64_t v = 0;
        memcpy(&v, p + i * s, s);
        nz = v != 0;
      }
    }
    local += nz ? 1 : 0;
  }
  for (int o = 16; o > 0; o >>= 1) local += __shfl_down_sync(0xffffffffu, local, o);
  if ((threadIdx.x & 31) == 0 && local) atomicAdd(count, local);
}

int op_count_nonzero(Arr *a, uint64_t *count) {
  Device *dev;
  SHLO_TRY(arr_device(a, &dev));
  Arr *c;
  SHLO_TRY(make_contiguous(a, &c));
  int64_t n = numel(c);
  Buffer *acc;
  int rc = buffer_alloc(dev, 8, &acc);
  if (!rc) {
    unsigned long long host = 0;
    rc = cuda_check(cudaMemsetAsync(acc->ptr, 0, 8, dev->stream), "count_nonzero");
    if (!rc && n > 0) {
      k_count_nonzero<<<grid_for(n, 256, dev), 256, 0, dev->stream>>>(data_ptr(c), c->dtype, n,
                                                                      (unsigned long long *)acc->ptr);
      rc = launch_check("count_nonzero");
    }
    if (!rc) rc = cuda_check(cudaMemcpyAsync(&host, acc->ptr, 8, cudaMemcpyDeviceToHost, dev->stream), "count_nonzero");
    if (!rc) rc = shlo_eval(&c, 1);
    *count = host;
    buffer_release(acc);
  }
  shlo_release(c);
  return rc;
}

// ------------------------------------------------------------ take ----

__global__ void k_take(int64_t outer, int64_t nidx, int64_t inner, int64_t len, const char *src, int esize,
                       const char *idx, int idt, char *dst) {
  int64_t n = outer * nidx * inner;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    int64_t in = i % inner;
    int64_t t = i / inner;
    int64_t j = t % nidx;
    int64_t o = t / nidx;
    int64_t k = load_as<int64_t>(idx, idt, j);
    if (idt == kU64) k = (int64_t)load_as<uint64_t>(idx, idt, j) >= len ? len - 1 : k;
    if (k < 0) k += len;
    k = k < 0 ? 0 : (k >= len ? len - 1 : k);
    int64_t s = (o * len + k) * inner + in;
    for (int b = 0; b < esize; b++) dst[i * esize + b] = src[s * esize + b];
  }
}

int op_take(Arr *a, Arr *idx, int axis, Arr **out) {
  if (axis < 0 || axis >= a->ndim) return fail("take: axis %d of a rank-%d array", axis, a->ndim);
  if (dtype_is_float(idx->dtype)) return fail("take: indices must be integers");
  if (a->shape[axis] == 0) return fail("take: empty axis");
  Device *dev;
  SHLO_TRY(arr_device(a, &dev));
  Arr *ca, *ci;
  SHLO_TRY(make_contiguous(a, &ca));
  if (make_contiguous(idx, &ci)) {
    shlo_release(ca);
    return 1;
  }
  int64_t outer = 1, inner = 1;
  for (int d = 0; d < axis; d++) outer *= a->shape[d];
  for (int d = axis + 1; d < a->ndim; d++) inner *= a->shape[d];
  int64_t shape[kMaxRank];
  int nd = 0;
  int rc = 0;
  if (a->ndim - 1 + idx->ndim > kMaxRank) rc = fail("take: result rank above %d", kMaxRank);
  for (int d = 0; d < axis && !rc; d++) shape[nd++] = a->shape[d];
  for (int d = 0; d < idx->ndim && !rc; d++) shape[nd++] = idx->shape[d];
  for (int d = axis + 1; d < a->ndim && !rc; d++) shape[nd++] = a->shape[d];
  Arr *o = nullptr;
  if (!rc) rc = new_array(dev, a->dtype, shape, nd, &o);
  int64_t nidx = numel(ci);
  if (!rc && outer * nidx * inner > 0) {
    k_take<<<grid_for(outer * nidx * inner, 256, dev), 256, 0, dev->stream>>>(
        outer, nidx, inner, a->shape[axis], data_ptr(ca), (int)dtype_size(a->dtype), data_ptr(ci), ci->dtype,
        (char *)o->buf->ptr);
    rc = launch_check("take");
  }
  shlo_release(ca);
  shlo_release(ci);
  if (rc) {
    if (o) shlo_release(o);
    return 1;
  }
  *out = o;
  return 0;
}

// ------------------------------------------------------------ concat ----

int op_concat(Arr *const *xs, int n, int axis, Arr **out) {
  if (n < 1) return fail("concatenate: no arrays");
  int nd = xs[0]->ndim;
  if (axis < 0 || axis >= nd) return fail("concatenate: axis %d of rank %d", axis, nd);
  int dt = xs[0]->dtype;
  int64_t shape[kMaxRank];
  for (int d = 0; d < nd; d++) shape[d] = xs[0]->shape[d];
  for (int i = 1; i < n; i++) {
    if (xs[i]->ndim != nd) return fail("concatenate: ranks differ");
    for (int d = 0; d < nd; d++)
      if (d != axis && xs[i]->shape[d] != shape[d]) return fail("concatenate: shapes differ off the axis");
    shape[axis] += xs[i]->shape[axis];
    dt = promote_types(dt, xs[i]->dtype);
  }
  Device *dev;
  SHLO_TRY(arr_device(xs[0], &dev));
  Arr *o;
  SHLO_TRY(new_array(dev, (uint8_t)dt, shape, nd, &o));
  int64_t at = 0;
  for (int i = 0; i < n; i++) {
    Arr *c;
    if (cast_array(xs[i], (uint8_t)dt, &c)) {
      shlo_release(o);
      return 1;
    }
    char *dst = (char *)o->buf->ptr + at * o->strides[axis] * (int64_t)dtype_size(dt);
    int rc = copy_into(dev, c, dst, o->strides);
    shlo_release(c);
    if (rc) {
      shlo_release(o);
      return 1;
    }
    at += xs[i]->shape[axis];
  }
  *out = o;
  return 0;
}

// ------------------------------------------------------------ built-in matmul ----
// a [..., n, k] @ b [..., k, m]: one thread per output, one accumulator summed in
// plain k order with fused multiply-add. This is deliberately not ggml's order:
// the planted `dotBuiltin` fault of Tests/OpTests.lean:120 must give other bits.

__global__ void k_matmul_plain(int64_t batch, int64_t n, int64_t k, int64_t m, const float *a, int64_t sa,
                               const float *b, int64_t sb, float *y) {
  int64_t total = batch * n * m;
  int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    int64_t col = i % m, row = (i / m) % n, bt = i / (m * n);
    const float *ar = a + bt * sa + row * k;
    const float *bc = b + bt * sb + col;
    float acc = 0.0f;
    for (int64_t t = 0; t < k; t++) acc = __fmaf_rn(ar[t], bc[t * m], acc);
    y[i] = acc;
  }
}

static int builtin_matmul(Arr *a, Arr *b, Arr **out) {
  if (a->ndim < 2 || b->ndim < 2) return fail("matmul: operands of rank below 2 not carried");
  if (!dtype_is_float(a->dtype) || !dtype_is_float(b->dtype)) return fail("matmul: integer operands not carried");
  int64_t n = a->shape[a->ndim - 2], k = a->shape[a->ndim - 1];
  int64_t k2 = b->shape[b->ndim - 2], m = b->shape[b->ndim - 1];
  if (k != k2) return fail("matmul: inner dimensions %lld and %lld", (long long)k, (long long)k2);
  int64_t bshape[kMaxRank];
  int bnd;
  SHLO_TRY(broadcast_shapes(a->shape, a->ndim - 2, b->shape, b->ndim - 2, bshape, &bnd));
  int64_t batch = 1;
  for (int d = 0; d < bnd; d++) batch *= bshape[d];
  int64_t sa_shape[kMaxRank], sb_shape[kMaxRank];
  for (int d = 0; d < bnd; d++) sa_shape[d] = sb_shape[d] = bshape[d];
  sa_shape[bnd] = n; sa_shape[bnd + 1] = k;
  sb_shape[bnd] = k; sb_shape[bnd + 1] = m;
  Device *dev;
  SHLO_TRY(arr_device(a, &dev));
  Arr *fa = nullptr, *fb = nullptr, *va = nullptr, *vb = nullptr, *ca = nullptr, *cb = nullptr, *o = nullptr;
  int rc = cast_array(a, kF32, &fa) || cast_array(b, kF32, &fb) || broadcast_view(fa, sa_shape, bnd + 2, &va) ||
           broadcast_view(fb, sb_shape, bnd + 2, &vb) || make_contiguous(va, &ca) || make_contiguous(vb, &cb);
  int64_t oshape[kMaxRank];
  for (int d = 0; d < bnd; d++) oshape[d] = bshape[d];
  oshape[bnd] = n;
  oshape[bnd + 1] = m;
  if (!rc) rc = new_array(dev, (uint8_t)promote_types(a->dtype, b->dtype), oshape, bnd + 2, &o);
  Arr *of = nullptr;
  if (!rc) rc = new_array(dev, kF32, oshape, bnd + 2, &of);
  if (!rc && batch * n * m > 0) {
    k_matmul_plain<<<grid_for(batch * n * m, 256, dev), 256, 0, dev->stream>>>(
        batch, n, k, m, (const float *)data_ptr(ca), n * k, (const float *)data_ptr(cb), k * m, (float *)of->buf->ptr);
    rc = launch_check("matmul");
  }
  Arr *res = nullptr;
  if (!rc) rc = cast_array(of, o->dtype, &res);
  for (Arr *t : {fa, fb, va, vb, ca, cb, o, of})
    if (t) shlo_release(t);
  if (rc) return 1;
  *out = res;
  return 0;
}

}  // namespace shlo

using namespace shlo;

// Each entry point below reads array data, so it opens a TraceScope (the op
// log of a compiled function's recording; see fusion.cu). Only the binary ops
// take part in fusions; the others are logged as uses of their inputs.
namespace {
enum OtherOp { OT_UNARY = 1, OT_WHERE, OT_ASTYPE, OT_TAKE, OT_MAX_AXIS, OT_CONCAT, OT_COUNT_NONZERO };

int traced(int kind, int sub, Arr *const *ins, int n, Arr **out, const std::function<int()> &run) {
  TraceScope ts(kind, sub, nullptr, 0, ins, n);
  if (ts.substituted()) return out ? ts.take(out) : fail("internal: a substituted op without a result");
  const int rc = run();
  if (!rc) ts.done(out ? *out : nullptr);
  return rc;
}
}  // namespace

extern "C" {

int shlo_unary(uint32_t op, shlo_arr a, shlo_arr *out) {
  if (!a) return fail("unary: null array");
  return traced(TK_OTHER, OT_UNARY, &a, 1, out, [&] { return op_unary(op, a, out); });
}
int shlo_binary(uint32_t op, shlo_arr a, shlo_arr b, shlo_arr *out) {
  if (!a || !b) return fail("binary: null array");
  Arr *ins[2] = {a, b};
  return traced(TK_BINARY, (int)op, ins, 2, out, [&] { return op_binary(op, a, b, out); });
}
int shlo_where(shlo_arr c, shlo_arr a, shlo_arr b, shlo_arr *out) {
  if (!c || !a || !b) return fail("where: null array");
  Arr *ins[3] = {c, a, b};
  return traced(TK_OTHER, OT_WHERE, ins, 3, out, [&] { return op_where(c, a, b, out); });
}
int shlo_astype(shlo_arr a, uint8_t dtype, shlo_arr *out) {
  if (!a) return fail("astype: null array");
  return traced(TK_OTHER, OT_ASTYPE, &a, 1, out, [&] { return op_astype(a, dtype, out); });
}
int shlo_take(shlo_arr a, shlo_arr idx, uint32_t axis, shlo_arr *out) {
  if (!a || !idx) return fail("take: null array");
  Arr *ins[2] = {a, idx};
  return traced(TK_OTHER, OT_TAKE, ins, 2, out, [&] { return op_take(a, idx, (int)axis, out); });
}
int shlo_max_axis(shlo_arr a, uint32_t axis, shlo_arr *out) {
  if (!a) return fail("max_axis: null array");
  return traced(TK_OTHER, OT_MAX_AXIS, &a, 1, out, [&] { return op_max_axis(a, (int)axis, out); });
}
int shlo_concat(const shlo_arr *xs, int n, uint32_t axis, shlo_arr *out) {
  for (int i = 0; i < n; i++)
    if (!xs[i]) return fail("concatenate: null array");
  Arr *const *ins = const_cast<Arr *const *>(xs);
  return traced(TK_OTHER, OT_CONCAT, ins, n, out, [&] { return op_concat(ins, n, (int)axis, out); });
}
int shlo_count_nonzero(shlo_arr a, uint64_t *count) {
  if (!a) return fail("count_nonzero: null array");
  return traced(TK_OTHER, OT_COUNT_NONZERO, &a, 1, nullptr, [&] { return op_count_nonzero(a, count); });
}

}  // extern "C"
