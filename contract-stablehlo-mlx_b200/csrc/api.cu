// The kernel and traced-function entry points of the boundary
// (c/smlx_shim.c:275-386) and the test-driver helpers (:388-414).
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <functional>
#include <vector>

#include "common.cuh"
#include "erff_cr.cuh"

using namespace shlo;

namespace {

enum KernelKind {
  KK_MUL_MAT, KK_SOFT_MAX, KK_NORM, KK_SILU, KK_GELU_ERF, KK_ERFF_MAP, KK_DIVIDE, KK_SQRT, KK_F64_EW,
  KK_F64_OF_F32, KK_F32_OF_F64
};

struct KernelInfo {
  const char *name;
  KernelKind kind;
  int n_inputs;     // binding order of StablehloMlx/Kernels/Shaders.lean
  int param_index;  // which input holds the parameter words
  int n_params;     // words read
  uint8_t out_dtype;
};

const KernelInfo kKernels[] = {
    {"smlx_mul_mat", KK_MUL_MAT, 3, 2, 6, kF32},       // w, x, p = [K, M, R, wbs, N, plain]
    {"smlx_soft_max", KK_SOFT_MAX, 2, 1, 4, kF32},     // x, p = [ncols, rows, scale bits, floatSum]
    {"smlx_norm", KK_NORM, 2, 1, 4, kF32},             // x, p = [ncols, rows, eps bits, gpuOps]
    {"smlx_silu", KK_SILU, 2, 1, 2, kF32},             // x, p = [count, gpuOps]
    {"smlx_gelu_erf", KK_GELU_ERF, 3, 2, 2, kF32},     // x, erffTable (unused), p = [count, gpuErf]
    {"smlx_erff_map", KK_ERFF_MAP, 2, 1, 2, kU32},     // erffTable (unused), p = [base, count]
    {"smlx_divide", KK_DIVIDE, 3, 2, 1, kF32},         // a, b, p = [count]
    {"smlx_sqrt", KK_SQRT, 2, 1, 1, kF32},             // a, p = [count]
    {"smlx_f64_ew", KK_F64_EW, 3, 2, 2, kU64},         // a, b, p = [count, op]
    {"smlx_f64_of_f32", KK_F64_OF_F32, 2, 1, 1, kU64}, // a, p = [count]
    {"smlx_f32_of_f64", KK_F32_OF_F64, 2, 1, 1, kF32}, // a, p = [count]
};

}  // namespace

struct shlo_kernel_s {
  const KernelInfo *info;
};

struct shlo_fn_s {
  shlo_trace_fn f;
  void *payload;
  void (*payload_free)(void *);
  int enable;
};

extern "C" {

int shlo_kernel_new(const char *name, const char *const *inputs, int n_inputs, const char *const *outputs,
                    int n_outputs, const char *source, const char *header, shlo_kernel *out) {
  (void)inputs; (void)outputs; (void)source; (void)header;
  if (!name) return fail("kernel: no name");
  for (const KernelInfo &k : kKernels) {
    if (strcmp(k.name, name) == 0) {
      if (n_inputs >= 0 && n_inputs != k.n_inputs)
        return fail("kernel %s: %d input names, %d expected", name, n_inputs, k.n_inputs);
      if (n_outputs >= 0 && n_outputs != 1) return fail("kernel %s: one output expected", name);
      shlo_kernel_s *h = new shlo_kernel_s();
      h->info = &k;
      *out = h;
      return 0;
    }
  }
  return fail("kernel %s: no such kernel in this backend (not carried)", name);
}

void shlo_kernel_free(shlo_kernel k) { delete k; }

int shlo_kernel_apply(shlo_kernel k, const shlo_arr *inputs, int n_inputs, const int64_t *const *out_shapes,
                      const int *out_ndims, const uint8_t *out_dtypes, int n_outputs, const int64_t grid[3],
                      const int64_t threadgroup[3], shlo_arr *outs) {
  (void)grid; (void)threadgroup;
  if (!k) return fail("kernel apply: null kernel");
  const KernelInfo &ki = *k->info;
  if (n_inputs != ki.n_inputs) return fail("kernel %s: %d inputs, %d expected", ki.name, n_inputs, ki.n_inputs);
  if (n_outputs != 1) return fail("kernel %s: one output expected", ki.name);
  for (int i = 0; i < n_inputs; i++)
    if (!inputs[i]) return fail("kernel %s: input %d is null", ki.name, i);
  if (out_dtypes[0] != ki.out_dtype)
    return fail("kernel %s: output dtype %s, %s expected", ki.name, dtype_name(out_dtypes[0]), dtype_name(ki.out_dtype));
  uint32_t p[8] = {0};
  SHLO_TRY(read_words(inputs[ki.param_index], p, ki.n_params));
  Device *dev;
  SHLO_TRY(arr_device(inputs[0], &dev));
  // The kernels index flat row-major buffers (c/smlx_shim.c:292-293).
  Arr *in[3] = {nullptr, nullptr, nullptr};
  int rc = 0;
  for (int i = 0; i < n_inputs && !rc; i++) {
    if (i == ki.param_index) continue;
    if (inputs[i]->buf && inputs[i]->buf->dev != dev) rc = fail("kernel %s: inputs on two devices", ki.name);
    else rc = make_contiguous(inputs[i], &in[i]);
    // Kernels read with 16-byte vector loads: an offset view gets its own copy.
    if (!rc && in[i]->buf && ((uintptr_t)data_ptr(in[i]) & 15)) {
      Arr *c = nullptr;
      rc = new_array(dev, in[i]->dtype, in[i]->shape, in[i]->ndim, &c);
      if (!rc) rc = launch_copy_strided(dev, in[i], c->buf->ptr);
      shlo_release(in[i]);
      in[i] = rc ? nullptr : c;
      if (rc && c) shlo_release(c);
    }
  }
  Arr *o = nullptr;
  if (!rc) {
    switch (ki.kind) {
      case KK_MUL_MAT: rc = k_mul_mat(dev, in[0], in[1], p, &o); break;
      case KK_SOFT_MAX: rc = k_soft_max(dev, in[0], p, &o); break;
      case KK_NORM: rc = k_norm(dev, in[0], p, &o); break;
      case KK_SILU: rc = k_silu(dev, in[0], p, &o); break;
      case KK_GELU_ERF: rc = k_gelu_erf(dev, in[0], p, &o); break;
      case KK_ERFF_MAP: rc = k_erff_map(dev, p, &o); break;
      case KK_DIVIDE: rc = k_divide(dev, in[0], in[1], p, &o); break;
      case KK_SQRT: rc = k_sqrt(dev, in[0], p, &o); break;
      case KK_F64_EW: rc = k_f64_ew(dev, in[0], in[1], p, &o); break;
      case KK_F64_OF_F32: rc = k_f64_of_f32(dev, in[0], p, &o); break;
      case KK_F32_OF_F64: rc = k_f32_of_f64(dev, in[0], p, &o); break;
    }
  }
  for (Arr *a : in)
    if (a) shlo_release(a);
  if (rc) return 1;
  // The requested output shape: the same element count, row-major.
  int64_t want = 1;
  for (int i = 0; i < out_ndims[0]; i++) want *= out_shapes[0][i];
  if (want != numel(o)) {
    int64_t got = numel(o);
    shlo_release(o);
    return fail("kernel %s: output shape of %lld elements, the parameters give %lld", ki.name, (long long)want,
                (long long)got);
  }
  rc = shlo_reshape(o, out_shapes[0], out_ndims[0], &outs[0]);
  shlo_release(o);
  return rc;
}

int shlo_compile(shlo_trace_fn f, void *payload, void (*payload_free)(void *), int enable, shlo_fn *out) {
  if (!f) return fail("compile: null function");
  shlo_fn_s *h = new shlo_fn_s();
  h->f = f;
  h->payload = payload;
  h->payload_free = payload_free;
  h->enable = enable;
  *out = h;
  return 0;
}

void shlo_fn_free(shlo_fn f) {
  if (!f) return;
  if (f->payload_free) f->payload_free(f->payload);
  delete f;
}

int shlo_apply(shlo_fn f, const shlo_arr *inputs, int n_inputs, shlo_arr *outputs, int *n_outputs, int max_outputs) {
  if (!f) return fail("apply: null function");
  char err[2048];
  err[0] = 0;
  int n = 0;
  int rc = f->f(f->payload, inputs, n_inputs, outputs, &n, max_outputs, err, sizeof err);
  if (rc) return fail("apply: traced function: %s", err[0] ? err : shlo_last_error());
  *n_outputs = n;
  return 0;
}

int shlo_libm_erff_range(uint32_t base, uint32_t count, uint32_t *out) {
  for (uint32_t i = 0; i < count; i++) {
    float x;
    uint32_t b = base + i;
    memcpy(&x, &b, 4);
    float y = shlo_erf::erff_cr(x);
    memcpy(&out[i], &y, 4);
  }
  return 0;
}

}  // extern "C"
