// The kernel and traced-function entry points of the boundary
// (c/smlx_shim.c:275-386) and the test-driver helpers (:388-414).
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <functional>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "erff_cr.cuh"

using namespace shlo;

namespace {

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
    // This backend's fused forms, which its executor uses in place of a kernel
    // followed by built-in adds and multiplies (the reference has none; every
    // rounding of the unfused sequence is kept):
    {"shlo_mul_mat_bias", KK_MUL_MAT_EP, 5, 4, 7, kF32},  // w, x, bias, residual, p = [mul_mat's six, flags]
    {"shlo_norm_affine", KK_NORM_AFFINE, 4, 3, 4, kF32},  // x, gamma, beta, p = [norm's four]
    {"shlo_attention", KK_ATTENTION, 4, 3, 5, kF32},      // q, k, v, p = [B, S, H, width, scale bits]
};

}  // namespace

struct shlo_kernel_s {
  const KernelInfo *info;
};

namespace {

// One recorded signature of a compiled function (Mlx.lean:66-67; mx::compile in
// c/smlx_shim.c:325-386). The graph reads private contiguous copies of the
// inputs (`staging`); a replay first refreshes the copies whose source array
// changed (arrays are immutable, so the same storage, offset and strides mean
// the same data), relaunches the graph, and copies the outputs into fresh
// arrays, so every result stays an independent immutable value.
struct Captured {
  bool eager = false;  // recording was refused for this signature: f runs every call
  std::string why;
  Device *dev = nullptr;
  std::vector<Arr *> staging;
  std::vector<Buffer *> src;        // source storage last copied into each slot (retained)
  std::vector<std::string> layout;  // and its offset, strides, dtype
  std::vector<Arr *> outs;          // the graph's results (its own storage)
  std::vector<std::pair<void *, size_t>> allocs;  // every block the graph owns
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  uint64_t launches = 0;  // kernel launches recorded in the graph
  int fused = 0;          // chains run as one fused launch each (fusion.cu)
};

std::string signature(Device *dev, const shlo_arr *inputs, int n) {
  std::string k = std::to_string(dev->id);
  for (int i = 0; i < n; i++) {
    k += "|";
    k += std::to_string((int)inputs[i]->dtype);
    for (int d = 0; d < inputs[i]->ndim; d++) k += "," + std::to_string((long long)inputs[i]->shape[d]);
  }
  return k;
}

std::string layout_of(const Arr *a) {
  std::string k = std::to_string((long long)a->offset) + ":" + std::to_string((int)a->dtype);
  for (int d = 0; d < a->ndim; d++) k += "," + std::to_string((long long)a->strides[d]);
  return k;
}

}  // namespace

struct shlo_fn_s {
  shlo_trace_fn f;
  void *payload;
  void (*payload_free)(void *);
  int enable;
  std::mutex mu;
  std::map<std::string, Captured *> graphs;
};

namespace {

int call_traced(shlo_fn f, const shlo_arr *inputs, int n_inputs, shlo_arr *outputs, int *n_outputs, int max_outputs) {
  char err[2048];
  err[0] = 0;
  int n = 0;
  int rc = f->f(f->payload, inputs, n_inputs, outputs, &n, max_outputs, err, sizeof err);
  if (rc) return fail("apply: traced function: %s", err[0] ? err : shlo_last_error());
  *n_outputs = n;
  return 0;
}

void release_all(shlo_arr *xs, int n) {
  for (int i = 0; i < n; i++)
    if (xs[i]) shlo_release(xs[i]);
}

void destroy_captured(Captured *c) {
  if (!c) return;
  if (c->dev) device_wait(c->dev, "compiled function free");
  if (c->exec) cudaGraphExecDestroy(c->exec);
  if (c->graph) cudaGraphDestroy(c->graph);
  for (Arr *a : c->outs) shlo_release(a);
  for (Arr *a : c->staging) shlo_release(a);
  for (Buffer *b : c->src) buffer_release(b);
  if (c->dev) {
    std::lock_guard<std::mutex> lk(c->dev->mu);
    for (auto &pb : c->allocs) {
      c->dev->free_blocks.emplace(pb.second, pb.first);
      c->dev->pooled_bytes += pb.second;
    }
  }
  delete c;
}

// Copy input i into its private slot when its source changed since the last
// call (and derive the slot's cached layouts again).
int refresh_slot(Captured *c, int i, Arr *in) {
  Arr *st = c->staging[i];
  if (!st->buf) return 0;
  const std::string lay = layout_of(in);
  if (in->buf == c->src[i] && lay == c->layout[i]) return 0;
  SHLO_TRY(launch_copy_strided(c->dev, in, st->buf->ptr));
  SHLO_TRY(buffer_rederive(st->buf));
  buffer_retain(in->buf);
  buffer_release(c->src[i]);
  c->src[i] = in->buf;
  c->layout[i] = lay;
  return 0;
}

// Record f over private copies of `inputs`. Returns nonzero only when f itself
// fails; a refusal to record (an operation that cannot run inside a graph)
// leaves c->eager set and f is then called eagerly for this signature.
int record(shlo_fn f, Device *dev, const shlo_arr *inputs, int n_inputs, int max_outputs, Captured *c) {
  c->dev = dev;
  for (int i = 0; i < n_inputs; i++) {
    Arr *in = inputs[i];
    Arr *st;
    SHLO_TRY(new_array(dev, in->dtype, in->shape, in->ndim, &st));
    c->staging.push_back(st);
    c->src.push_back(nullptr);
    c->layout.push_back("");
    SHLO_TRY(refresh_slot(c, i, in));
  }
  // One eager call first: it derives every cached layout of the inputs (the
  // packed weights of mul_mat) outside the graph, and checks f. Its ops are
  // logged; the fused chains found in the log run as one launch each in the
  // capture call (fusion.cu).
  std::unique_ptr<Tracer, void (*)(Tracer *)> tr(fusion_enabled() ? tracer_new(dev) : nullptr, tracer_free);
  {
    std::vector<shlo_arr> tmp(max_outputs > 0 ? max_outputs : 1, nullptr);
    int n = 0;
    Tracer *outer = t_tracer;  // a recording in progress around this one (a nested compiled function)
    t_tracer = tr.get();
    const int frc = call_traced(f, c->staging.data(), n_inputs, tmp.data(), &n, max_outputs);
    t_tracer = outer;
    SHLO_TRY(frc);
    if (tr) c->fused = tracer_plan(tr.get(), tmp.data(), n);
    release_all(tmp.data(), n);
    if (tr && c->fused == 0) tr.reset();
  }
  // Nothing queued may still use a pooled block once the recording claims it.
  SHLO_TRY(device_wait(dev, "compile"));
  std::vector<shlo_arr> outs(max_outputs > 0 ? max_outputs : 1, nullptr);
  int n_out = 0;
  const uint64_t l0 = g_launches.load();
  cudaError_t e = cudaStreamBeginCapture(dev->stream, cudaStreamCaptureModeRelaxed);
  if (e != cudaSuccess) {
    cudaGetLastError();
    c->eager = true;
    c->why = std::string("begin capture: ") + cudaGetErrorString(e);
    return 0;
  }
  {
    std::lock_guard<std::mutex> lk(dev->mu);
    dev->capturing = true;
    dev->capture_owner = c;
    dev->capture_allocs = &c->allocs;
  }
  Tracer *outer = t_tracer;
  t_tracer = tr.get();
  int frc = call_traced(f, c->staging.data(), n_inputs, outs.data(), &n_out, max_outputs);
  t_tracer = outer;
  std::string ferr = frc ? shlo_last_error() : "";
  std::string unfused;
  if (!frc && tr && !tracer_complete(tr.get(), &unfused)) {
    frc = 1;  // the capture call departed from the eager call: record nothing, run unfused
    ferr = "fusion: " + unfused;
  }
  cudaGraph_t g = nullptr;
  e = cudaStreamEndCapture(dev->stream, &g);
  c->launches = g_launches.load() - l0;
  {
    std::lock_guard<std::mutex> lk(dev->mu);
    dev->capturing = false;
    dev->capture_owner = nullptr;
    dev->capture_allocs = nullptr;
    dev->capture_free.clear();  // the graph keeps these blocks (in c->allocs)
  }
  if (e == cudaSuccess && !frc) e = cudaGraphInstantiate(&c->exec, g, 0);
  if (frc || e != cudaSuccess) {
    cudaGetLastError();
    release_all(outs.data(), n_out);
    if (g) cudaGraphDestroy(g);
    c->exec = nullptr;
    c->eager = true;
    c->why = frc ? "traced function inside a capture: " + ferr : std::string("capture: ") + cudaGetErrorString(e);
    return 0;
  }
  c->graph = g;
  c->outs.assign(outs.begin(), outs.begin() + n_out);
  return 0;
}

}  // namespace

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
  // The op log of a compiled function's recording (fusion.cu): in the capture
  // call an op of a fused chain returns its substitute here.
  TraceScope ts(TK_KERNEL, (int)ki.kind, p, ki.n_params, inputs, n_inputs);
  if (ts.substituted()) return ts.take(&outs[0]);
  Device *dev;
  SHLO_TRY(arr_device(inputs[0], &dev));
  // The kernels index flat row-major buffers (c/smlx_shim.c:292-293).
  Arr *in[5] = {nullptr, nullptr, nullptr, nullptr, nullptr};
  int rc = 0;
  for (int i = 0; i < n_inputs && !rc; i++) {
    if (i == ki.param_index) continue;
    if (inputs[i]->buf && inputs[i]->buf->dev != dev) {
      rc = fail("kernel %s: inputs on two devices", ki.name);
      break;
    }
    if (ki.kind == KK_ATTENTION) {  // reads strided views itself (and copies what it cannot)
      inputs[i]->rc.fetch_add(1);
      in[i] = inputs[i];
      continue;
    }
    rc = make_contiguous(inputs[i], &in[i]);
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
      case KK_MUL_MAT_EP: rc = k_mul_mat_ep(dev, in[0], in[1], p, in[2], in[3], (int)p[6], &o); break;
      case KK_NORM_AFFINE: rc = k_norm_affine(dev, in[0], p, in[1], in[2], &o); break;
      case KK_ATTENTION: rc = k_attention(dev, in[0], in[1], in[2], p, &o); break;
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
  if (!rc) ts.done(outs[0]);
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
  for (auto &kv : f->graphs) destroy_captured(kv.second);
  if (f->payload_free) f->payload_free(f->payload);
  delete f;
}

int shlo_apply(shlo_fn f, const shlo_arr *inputs, int n_inputs, shlo_arr *outputs, int *n_outputs, int max_outputs) {
  if (!f) return fail("apply: null function");
  for (int i = 0; i < n_inputs; i++)
    if (!inputs[i]) return fail("apply: input %d is null", i);
  if (!f->enable) return call_traced(f, inputs, n_inputs, outputs, n_outputs, max_outputs);
  Device *dev;
  // No device to record on: the function runs as called (its own ops report
  // the error, if it has any).
  if (current_device(&dev)) return call_traced(f, inputs, n_inputs, outputs, n_outputs, max_outputs);
  if (dev->capturing) return call_traced(f, inputs, n_inputs, outputs, n_outputs, max_outputs);  // nested
  std::lock_guard<std::mutex> lk(f->mu);
  const std::string key = signature(dev, inputs, n_inputs);
  Captured *c;
  auto it = f->graphs.find(key);
  if (it != f->graphs.end()) {
    c = it->second;
  } else {
    c = new Captured();
    if (record(f, dev, inputs, n_inputs, max_outputs, c)) {
      std::string msg = shlo_last_error();
      destroy_captured(c);
      return fail("%s", msg.c_str());
    }
    f->graphs[key] = c;
    if (getenv("SHLO_GRAPH_VERBOSE")) {
      if (c->eager)
        fprintf(stderr, "shlo: compiled function runs eagerly: %s\n", c->why.c_str());
      else
        fprintf(stderr, "shlo: compiled function recorded: %llu launches, %d fused chains\n",
                (unsigned long long)c->launches, c->fused);
    }
  }
  if (c->eager) return call_traced(f, inputs, n_inputs, outputs, n_outputs, max_outputs);
  if ((int)c->outs.size() > max_outputs) return fail("apply: %d outputs, room for %d", (int)c->outs.size(), max_outputs);
  for (int i = 0; i < n_inputs; i++) {
    if (inputs[i]->buf && inputs[i]->buf->dev != dev) return fail("apply: input %d is on another device", i);
    SHLO_TRY(refresh_slot(c, i, inputs[i]));
  }
  SHLO_CUDA(cudaGraphLaunch(c->exec, dev->stream));
  g_launches.fetch_add(c->launches, std::memory_order_relaxed);
  int n = 0;
  for (Arr *o : c->outs) {
    Arr *r;
    int rc = new_array(dev, o->dtype, o->shape, o->ndim, &r);
    if (!rc && r->buf) rc = launch_copy_strided(dev, o, r->buf->ptr);
    // a result is often read back at once, while the next call computes
    if (!rc && r->buf && !dev->capturing)
      rc = cuda_check(cudaEventCreateWithFlags(&r->buf->ready, cudaEventDisableTiming), "apply") ||
           cuda_check(cudaEventRecord(r->buf->ready, dev->stream), "apply");
    if (rc) {
      if (r) shlo_release(r);
      release_all(outputs, n);
      return 1;
    }
    outputs[n++] = r;
  }
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
