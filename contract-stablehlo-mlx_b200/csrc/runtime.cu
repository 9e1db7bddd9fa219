// shlo_cuda runtime: devices, storage, array handles, views, readback, eval.
//
// Replaces the mlx-c plumbing of the reference shim (c/smlx_shim.c:15-139,
// 203-273): one non-blocking CUDA stream per device stands in for MLX's
// default GPU stream, arrays are reference-counted immutable values over
// pooled device storage, and transpose/broadcast/slice are strided views.
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <thread>

#include "common.cuh"

namespace shlo {

// ---------------------------------------------------------------- errors ----

static thread_local std::string t_error;

int fail(const char *fmt, ...) {
  char buf[2048];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  t_error = buf;
  return 1;
}

int cuda_check(cudaError_t e, const char *what) {
  if (e == cudaSuccess) return 0;
  return fail("%s: CUDA error %d (%s)", what, (int)e, cudaGetErrorString(e));
}

std::atomic<uint64_t> g_launches{0};

int launch_check(const char *what) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return cuda_check(cudaGetLastError(), what);
}

// ---------------------------------------------------------------- dtypes ----

static const size_t kSizes[kNumDTypes] = {1, 1, 2, 4, 8, 1, 2, 4, 8, 2, 4};
static const char *kNames[kNumDTypes] = {"bool", "uint8", "uint16", "uint32", "uint64", "int8",
                                         "int16", "int32", "int64", "float16", "float32"};
bool dtype_valid(int dt) { return dt >= 0 && dt < kNumDTypes; }
size_t dtype_size(int dt) { return dtype_valid(dt) ? kSizes[dt] : 0; }
const char *dtype_name(int dt) { return dtype_valid(dt) ? kNames[dt] : "?"; }
bool dtype_is_float(int dt) { return dt == kF16 || dt == kF32; }
bool dtype_is_signed_int(int dt) { return dt == kI8 || dt == kI16 || dt == kI32 || dt == kI64; }
bool dtype_is_unsigned_int(int dt) { return dt == kU8 || dt == kU16 || dt == kU32 || dt == kU64; }

// MLX's type promotion (mlx/dtype.cpp, promote_types) restricted to these dtypes:
// bool < unsigned/signed integers < float16 < float32; mixing signed and unsigned
// widens to the next signed type; uint64 with any signed integer gives float32.
int promote_types(int a, int b) {
  if (a == b) return a;
  if (a == kBool) return b;
  if (b == kBool) return a;
  if (dtype_is_float(a) || dtype_is_float(b)) {
    if (a == kF32 || b == kF32) return kF32;
    return kF16;
  }
  auto bits = [](int t) { return (int)dtype_size(t) * 8; };
  bool ua = dtype_is_unsigned_int(a), ub = dtype_is_unsigned_int(b);
  if (ua == ub) return bits(a) >= bits(b) ? a : b;
  int u = ua ? a : b, s = ua ? b : a;
  if (u == kU64) return kF32;
  int need = bits(u) * 2 > bits(s) ? bits(u) * 2 : bits(s);
  switch (need) {
    case 8: return kI8;
    case 16: return kI16;
    case 32: return kI32;
    default: return kI64;
  }
}

// --------------------------------------------------------------- devices ----

static std::mutex g_dev_mu;
static Device *g_devs[64];
static thread_local int t_device = -1;
static thread_local int t_cuda_set = -1;
static std::atomic<int> g_flavor{-1};

static int init_device(int id, Device **out) {
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (id < 0 || id >= 64) return fail("device %d out of range", id);
  if (!g_devs[id]) {
    int n = 0;
    SHLO_CUDA(cudaGetDeviceCount(&n));
    if (id >= n) return fail("device %d: only %d CUDA devices", id, n);
    SHLO_CUDA(cudaSetDevice(id));
    Device *d = new Device();
    d->id = id;
    SHLO_CUDA(cudaDeviceGetAttribute(&d->sm_count, cudaDevAttrMultiProcessorCount, id));
    SHLO_CUDA(cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking));
    SHLO_CUDA(cudaStreamCreateWithFlags(&d->copy, cudaStreamNonBlocking));
    SHLO_CUDA(cudaHostAlloc((void **)&d->pipe_err_host, sizeof(int), cudaHostAllocMapped));
    *d->pipe_err_host = 0;
    SHLO_CUDA(cudaHostGetDevicePointer((void **)&d->pipe_err_dev, d->pipe_err_host, 0));
    g_devs[id] = d;
  }
  *out = g_devs[id];
  return 0;
}

int device_by_id(int id, Device **out) {
  SHLO_TRY(init_device(id, out));
  if (t_cuda_set != id) {
    SHLO_CUDA(cudaSetDevice(id));
    t_cuda_set = id;
  }
  return 0;
}

int current_device(Device **out) {
  if (t_device < 0) {
    const char *e = getenv("SHLO_DEVICE");
    t_device = e ? atoi(e) : 0;
  }
  return device_by_id(t_device, out);
}

int current_flavor() {
  int f = g_flavor.load();
  if (f < 0) {
    const char *e = getenv("SHLO_GGML_FLAVOR");
    f = (e && strcmp(e, "stock") == 0) ? 1 : 0;
    g_flavor.store(f);
  }
  return f;
}

// --------------------------------------------------------------- storage ----
// A caching allocator per device. Blocks freed by a release go back to the
// pool and may be handed to the next allocation at once: every use of device
// memory is ordered on the device's single stream, so the next user's kernels
// run after the last reader's.

static size_t round_bytes(size_t n) {
  if (n == 0) n = 1;
  return (n + 511) & ~(size_t)511;
}

static std::atomic<uint64_t> g_serial{0};
static uint64_t next_serial() { return g_serial.fetch_add(1) + 1; }

static int take_block(Device *dev, size_t want, bool from_capture, void **p, size_t *got) {
  *p = nullptr;
  *got = want;
  std::lock_guard<std::mutex> lk(dev->mu);
  if (from_capture) {
    auto it = dev->capture_free.lower_bound(want);
    if (it != dev->capture_free.end() && it->first <= want * 2 + 65536) {
      *got = it->first;
      *p = it->second;
      dev->capture_free.erase(it);
      return 1;  // already the graph's
    }
  }
  auto it = dev->free_blocks.lower_bound(want);
  if (it != dev->free_blocks.end() && it->first <= want * 2 + 65536) {
    *got = it->first;
    *p = it->second;
    dev->free_blocks.erase(it);
    dev->pooled_bytes -= *got;
  }
  return 0;
}

static int alloc_block(Device *dev, size_t bytes, bool constant, Buffer **out) {
  size_t want = round_bytes(bytes);
  void *p = nullptr;
  size_t got = want;
  const bool cap = dev->capturing && dev->capture_allocs;
  const int graphs = take_block(dev, want, cap && !constant, &p, &got);
  if (!p) {
    cudaError_t e = cudaMalloc(&p, want);
    if (e != cudaSuccess) {
      cudaGetLastError();
      // Out of memory: give the pool back and try once more (not while a
      // capture is recording: the stream cannot be waited on then).
      if (cap) return cuda_check(e, "cudaMalloc");
      std::lock_guard<std::mutex> lk(dev->mu);
      SHLO_CUDA(cudaStreamSynchronize(dev->stream));
      for (auto &kv : dev->free_blocks) cudaFree(kv.second);
      dev->free_blocks.clear();
      dev->pooled_bytes = 0;
      // idle upload blocks too (their release events are behind the synchronize)
      for (auto &kv : dev->upload_free) {
        if (kv.second.second) cudaEventDestroy(kv.second.second);
        cudaFree(kv.second.first);
      }
      dev->upload_free.clear();
      e = cudaMalloc(&p, want);
      if (e != cudaSuccess) return cuda_check(e, "cudaMalloc");
    }
  }
  Buffer *b = new Buffer();
  b->serial = next_serial();
  b->dev = dev;
  b->ptr = p;
  b->bytes = got;
  if (cap) {
    b->graph_owner = dev->capture_owner;
    b->no_recycle = constant;
    if (!graphs) dev->capture_allocs->push_back({p, got});
  }
  *out = b;
  return 0;
}

int buffer_alloc(Device *dev, size_t bytes, Buffer **out) { return alloc_block(dev, bytes, false, out); }

// A block for an upload of shlo_of_bytes on the copy stream. Upload blocks have
// a pool of their own: a block goes back to it with an event recorded on the
// compute stream when it is released (after every read of it queued so far),
// and the copy stream waits for that event alone before writing it again, so
// an upload never waits for unrelated compute.
static int alloc_upload(Device *dev, size_t bytes, Buffer **out) {
  const size_t want = round_bytes(bytes);
  void *p = nullptr;
  size_t got = want;
  cudaEvent_t ev = nullptr;
  {
    std::lock_guard<std::mutex> lk(dev->mu);
    auto it = dev->upload_free.lower_bound(want);
    if (it != dev->upload_free.end() && it->first <= want * 2 + 65536) {
      got = it->first;
      p = it->second.first;
      ev = it->second.second;
      dev->upload_free.erase(it);
    }
  }
  if (p) {
    cudaError_t e = cudaSuccess;
    if (!ev) {  // released without an event: after everything queued so far
      e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
      if (e == cudaSuccess) e = cudaEventRecord(ev, dev->stream);
    }
    if (e == cudaSuccess) e = cudaStreamWaitEvent(dev->copy, ev, 0);
    if (ev) cudaEventDestroy(ev);
    if (e != cudaSuccess) {
      cudaFree(p);
      return cuda_check(e, "ofBytes: upload block");
    }
  } else {
    SHLO_CUDA(cudaMalloc(&p, want));
  }
  Buffer *b = new Buffer();
  b->serial = next_serial();
  b->dev = dev;
  b->ptr = p;
  b->bytes = got;
  b->upload = true;
  *out = b;
  return 0;
}
int buffer_alloc_constant(Device *dev, size_t bytes, Buffer **out) { return alloc_block(dev, bytes, true, out); }

void buffer_retain(Buffer *b) {
  if (b) b->rc.fetch_add(1);
}

void buffer_release(Buffer *b) {
  if (!b) return;
  if (b->rc.fetch_sub(1) != 1) return;
  for (auto &kv : b->derived) buffer_release(kv.second);
  Device *dev = b->dev;
  // An upload block's release event (none while a capture records on the
  // stream: the next upload into the block then waits for the whole stream).
  cudaEvent_t freed = nullptr;
  if (b->upload && !dev->capturing &&
      (cudaEventCreateWithFlags(&freed, cudaEventDisableTiming) != cudaSuccess ||
       cudaEventRecord(freed, dev->stream) != cudaSuccess)) {
    cudaGetLastError();
    if (freed) cudaEventDestroy(freed);
    freed = nullptr;
  }
  {
    std::lock_guard<std::mutex> lk(dev->mu);
    if (b->upload) {
      dev->upload_free.emplace(b->bytes, std::make_pair(b->ptr, freed));
    } else if (!b->graph_owner) {
      dev->free_blocks.emplace(b->bytes, b->ptr);
      dev->pooled_bytes += b->bytes;
    } else if (dev->capturing && dev->capture_owner == b->graph_owner && !b->no_recycle) {
      dev->capture_free.emplace(b->bytes, b->ptr);
    }
  }
  if (b->ready) cudaEventDestroy(b->ready);
  delete b;
}

int buffer_rederive(Buffer *b) {
  std::lock_guard<std::mutex> lk(b->derived_mu);
  for (auto &kv : b->rederive)
    if (kv.second()) return 1;
  return 0;
}

// ---------------------------------------------------------------- arrays ----

int64_t numel(const Arr *a) {
  int64_t n = 1;
  for (int i = 0; i < a->ndim; i++) n *= a->shape[i];
  return n;
}

bool is_row_contiguous(const Arr *a) {
  int64_t s = 1;
  for (int i = a->ndim - 1; i >= 0; i--) {
    if (a->shape[i] != 1 && a->strides[i] != s) return false;
    s *= a->shape[i];
  }
  return true;
}

void set_row_major(Arr *a) {
  int64_t s = 1;
  for (int i = a->ndim - 1; i >= 0; i--) {
    a->strides[i] = s;
    s *= a->shape[i];
  }
}

int new_array(Device *dev, uint8_t dtype, const int64_t *shape, int ndim, Arr **out) {
  if (ndim < 0 || ndim > kMaxRank) return fail("rank %d above %d", ndim, kMaxRank);
  Arr *a = new Arr();
  a->dtype = dtype;
  a->ndim = ndim;
  for (int i = 0; i < ndim; i++) {
    if (shape[i] < 0) {
      delete a;
      return fail("negative dimension %lld", (long long)shape[i]);
    }
    a->shape[i] = shape[i];
  }
  set_row_major(a);
  size_t bytes = (size_t)numel(a) * dtype_size(dtype);
  if (buffer_alloc(dev, bytes, &a->buf)) {
    delete a;
    return 1;
  }
  *out = a;
  return 0;
}

Arr *new_view(const Arr *src) {
  Arr *a = new Arr();
  a->dtype = src->dtype;
  a->ndim = src->ndim;
  for (int i = 0; i < src->ndim; i++) {
    a->shape[i] = src->shape[i];
    a->strides[i] = src->strides[i];
  }
  a->offset = src->offset;
  a->buf = src->buf;
  buffer_retain(a->buf);
  return a;
}

int arr_device(const Arr *a, Device **out) {
  if (!a) return fail("null array");
  if (!a->buf) return current_device(out);
  return device_by_id(a->buf->dev->id, out);
}

static void release_arr(Arr *a) {
  if (!a) return;
  if (a->rc.fetch_sub(1) != 1) return;
  buffer_release(a->buf);
  delete a;
}

int make_contiguous(Arr *a, Arr **out) {
  if (is_row_contiguous(a) || !a->buf) {
    a->rc.fetch_add(1);
    *out = a;
    return 0;
  }
  Device *dev;
  SHLO_TRY(arr_device(a, &dev));
  Arr *c;
  SHLO_TRY(new_array(dev, a->dtype, a->shape, a->ndim, &c));
  if (launch_copy_strided(dev, a, c->buf->ptr)) {
    release_arr(c);
    return 1;
  }
  *out = c;
  return 0;
}

// Wait for all queued work on a device, bounded by SHLO_EVAL_TIMEOUT_S.
static int wait_stream(Device *dev, cudaStream_t stream, const char *what) {
  static double limit = [] {
    const char *e = getenv("SHLO_EVAL_TIMEOUT_S");
    return e ? atof(e) : 600.0;
  }();
  auto t0 = std::chrono::steady_clock::now();
  for (int spins = 0;; spins++) {
    cudaError_t e = cudaStreamQuery(stream);
    if (e == cudaSuccess) {
      volatile int *perr = dev->pipe_err_host;
      if (perr && *perr) {
        *perr = 0;
        return fail("%s: a mul_mat launch on device %d gave up waiting for its stage copies (the results are "
                    "not valid)", what, dev->id);
      }
      return 0;
    }
    if (e != cudaErrorNotReady) return cuda_check(e, what);
    double dt = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (dt > limit) return fail("%s: device %d did not finish within %.0f s", what, dev->id, limit);
    if (spins < 2000) std::this_thread::yield();
    else std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

static int wait_device(Device *dev, const char *what) { return wait_stream(dev, dev->stream, what); }

int device_wait(Device *dev, const char *what) { return wait_device(dev, what); }

int read_words(Arr *a, uint32_t *words, int n) {
  if ((int64_t)numel(a) * (int64_t)dtype_size(a->dtype) < (int64_t)n * 4)
    return fail("parameter array has %lld elements of %s, %d words needed", (long long)numel(a),
                dtype_name(a->dtype), n);
  if (a->has_host) {
    memcpy(words, a->host.data(), (size_t)n * 4);
    return 0;
  }
  // Computed on the device: read it back (a synchronous round trip).
  Device *dev;
  SHLO_TRY(arr_device(a, &dev));
  Arr *c;
  SHLO_TRY(make_contiguous(a, &c));
  cudaError_t e = cudaMemcpyAsync(words, data_ptr(c), (size_t)n * 4, cudaMemcpyDeviceToHost, dev->stream);
  int rc = cuda_check(e, "parameter readback") || wait_device(dev, "parameter readback");
  release_arr(c);
  return rc;
}

int broadcast_shapes(const int64_t *a, int na, const int64_t *b, int nb, int64_t *out, int *nout) {
  int n = na > nb ? na : nb;
  if (n > kMaxRank) return fail("broadcast rank %d above %d", n, kMaxRank);
  for (int i = 0; i < n; i++) {
    int64_t da = i < n - na ? 1 : a[i - (n - na)];
    int64_t db = i < n - nb ? 1 : b[i - (n - nb)];
    if (da != db && da != 1 && db != 1)
      return fail("shapes cannot be broadcast (axis %d: %lld vs %lld)", i, (long long)da, (long long)db);
    out[i] = da == 1 ? db : da;
  }
  *nout = n;
  return 0;
}

int broadcast_view(Arr *a, const int64_t *shape, int ndim, Arr **out) {
  if (ndim < a->ndim) return fail("broadcast: rank %d below the array's %d", ndim, a->ndim);
  if (ndim > kMaxRank) return fail("broadcast: rank %d above %d", ndim, kMaxRank);
  Arr *v = new_view(a);
  v->ndim = ndim;
  int off = ndim - a->ndim;
  for (int i = 0; i < ndim; i++) {
    int64_t src = i < off ? 1 : a->shape[i - off];
    int64_t st = i < off ? 0 : a->strides[i - off];
    if (src == shape[i]) {
      v->shape[i] = src;
      v->strides[i] = src == 1 ? 0 : st;
    } else if (src == 1) {
      v->shape[i] = shape[i];
      v->strides[i] = 0;
    } else {
      release_arr(v);
      return fail("broadcast: cannot broadcast axis %d of size %lld to %lld", i - off, (long long)src,
                  (long long)shape[i]);
    }
  }
  *out = v;
  return 0;
}

}  // namespace shlo

using namespace shlo;

// ================================================================= C ABI ====

extern "C" {

const char *shlo_last_error(void) { return t_error.c_str(); }

int shlo_set_device(int device) {
  Device *d;
  SHLO_TRY(init_device(device, &d));
  t_device = device;
  return device_by_id(device, &d);
}

int shlo_get_device(int *device) {
  Device *d;
  SHLO_TRY(current_device(&d));
  *device = d->id;
  return 0;
}

int shlo_device_count(int *count) {
  SHLO_CUDA(cudaGetDeviceCount(count));
  return 0;
}

int shlo_set_flavor(int flavor) {
  if (flavor != 0 && flavor != 1) return fail("flavor must be 0 (pinned) or 1 (stock)");
  g_flavor.store(flavor);
  return 0;
}

int shlo_get_flavor(int *flavor) {
  *flavor = current_flavor();
  return 0;
}

int shlo_current_stream(void **stream) {
  Device *d;
  SHLO_TRY(current_device(&d));
  *stream = (void *)d->stream;
  return 0;
}

int shlo_launch_count(uint64_t *count) {
  *count = g_launches.load();
  return 0;
}

int shlo_device_ptr(shlo_arr a, void **ptr, int *device) {
  if (!a) return fail("device_ptr: null array");
  TraceScope ts(TK_OTHER, 21, nullptr, 0, &a, 1);  // the data escapes to the caller
  ts.done(nullptr);
  if (!a->buf) return fail("device_ptr: the array has no storage");
  if (!is_row_contiguous(a)) return fail("device_ptr: the array is a strided view (make it contiguous first)");
  *ptr = data_ptr(a);
  if (device) *device = a->buf->dev->id;
  return 0;
}

void shlo_retain(shlo_arr a) {
  if (a) a->rc.fetch_add(1);
}

void shlo_release(shlo_arr a) { release_arr(a); }

shlo_arr shlo_empty(void) {
  Arr *a = new Arr();
  a->dtype = kF32;
  a->ndim = 1;
  a->shape[0] = 0;
  a->strides[0] = 1;
  return a;
}

int shlo_of_bytes(const void *data, size_t nbytes, const int64_t *shape, int ndim, uint8_t dtype,
                  shlo_arr *out) {
  if (ndim > kMaxRank) return fail("ofBytes: rank above %d", kMaxRank);
  if (!dtype_valid(dtype)) return fail("ofBytes: dtype %d not carried", (int)dtype);
  int64_t count = 1;
  for (int i = 0; i < ndim; i++) count *= shape[i];
  if ((size_t)count * dtype_size(dtype) != nbytes) return fail("ofBytes: byte count does not match the shape");
  Device *dev;
  SHLO_TRY(current_device(&dev));
  Arr *a;
  if (dev->capturing) {
    // Recording a compiled function: the data is a constant of the graph. It
    // is written now, synchronously, into a block the capture never reuses
    // (a copy on the recording stream would become a node reading this host
    // memory at every replay).
    a = new Arr();
    a->dtype = dtype;
    a->ndim = ndim;
    for (int i = 0; i < ndim; i++) a->shape[i] = shape[i];
    set_row_major(a);
    if (buffer_alloc_constant(dev, nbytes, &a->buf)) {
      delete a;
      return 1;
    }
    if (nbytes && cuda_check(cudaMemcpy(a->buf->ptr, data, nbytes, cudaMemcpyHostToDevice), "ofBytes (capture)")) {
      release_arr(a);
      return 1;
    }
    if (nbytes <= 256) {
      a->host.assign((const uint8_t *)data, (const uint8_t *)data + nbytes);
      a->has_host = true;
    }
    *out = a;
    return 0;
  }
  cudaPointerAttributes at;
  const bool pinned = nbytes && cudaPointerGetAttributes(&at, data) == cudaSuccess && at.type == cudaMemoryTypeHost;
  cudaGetLastError();
  if (pinned && nbytes > 256) {
    // A pinned input (above the size whose bytes are also kept on the host):
    // uploaded on the copy stream into an upload block, beside the compute
    // still queued (the host waits for the copy alone).
    a = new Arr();
    a->dtype = dtype;
    a->ndim = ndim;
    for (int i = 0; i < ndim; i++) a->shape[i] = shape[i];
    set_row_major(a);
    if (alloc_upload(dev, nbytes, &a->buf)) {
      delete a;
      return 1;
    }
    if (cuda_check(cudaMemcpyAsync(a->buf->ptr, data, nbytes, cudaMemcpyHostToDevice, dev->copy), "ofBytes") ||
        wait_stream(dev, dev->copy, "ofBytes")) {
      release_arr(a);
      return 1;
    }
    *out = a;
    return 0;
  }
  SHLO_TRY(new_array(dev, dtype, shape, ndim, &a));
  if (nbytes) {
    cudaError_t e = cudaMemcpyAsync(a->buf->ptr, data, nbytes, cudaMemcpyHostToDevice, dev->stream);
    if (e == cudaSuccess && pinned) e = cudaStreamSynchronize(dev->stream);  // consumed before return
    if (cuda_check(e, "ofBytes: host to device copy")) {
      release_arr(a);
      return 1;
    }
  }
  if (nbytes <= 256) {
    a->host.assign((const uint8_t *)data, (const uint8_t *)data + nbytes);
    a->has_host = true;
  }
  *out = a;
  return 0;
}

int shlo_nbytes(shlo_arr a, size_t *nbytes) {
  if (!a) return fail("null array");
  *nbytes = (size_t)numel(a) * dtype_size(a->dtype);
  return 0;
}

int shlo_to_bytes(shlo_arr a, void *dst, size_t cap) {
  if (!a) return fail("toBytes: null array");
  TraceScope ts(TK_OTHER, 20, nullptr, 0, &a, 1);  // a read of the array's data
  ts.done(nullptr);
  size_t bytes = (size_t)numel(a) * dtype_size(a->dtype);
  if (cap < bytes) return fail("toBytes: %zu bytes needed, %zu given", bytes, cap);
  if (bytes == 0) return 0;
  Device *dev;
  SHLO_TRY(arr_device(a, &dev));
  Arr *c;
  SHLO_TRY(make_contiguous(a, &c));
  int rc;
  if (dev->capturing) {
    rc = cuda_check(cudaMemcpyAsync(dst, data_ptr(c), bytes, cudaMemcpyDeviceToHost, dev->stream), "toBytes") ||
         wait_device(dev, "toBytes");
  } else {
    // On the copy stream, after the array's producer: its buffer's ready event
    // where it has one (a graph replay's result), so that work queued on the
    // compute stream after the producer runs on while the bytes cross to the
    // host; otherwise everything queued on the compute stream so far.
    cudaEvent_t ready = c->buf->ready, own = nullptr;
    rc = 0;
    if (!ready) {
      rc = cuda_check(cudaEventCreateWithFlags(&own, cudaEventDisableTiming), "toBytes") ||
           cuda_check(cudaEventRecord(own, dev->stream), "toBytes");
      ready = own;
    }
    if (!rc)
      rc = cuda_check(cudaStreamWaitEvent(dev->copy, ready, 0), "toBytes") ||
           cuda_check(cudaMemcpyAsync(dst, data_ptr(c), bytes, cudaMemcpyDeviceToHost, dev->copy), "toBytes") ||
           wait_stream(dev, dev->copy, "toBytes");
    if (own) cudaEventDestroy(own);
  }
  release_arr(c);
  return rc;
}

int shlo_shape(shlo_arr a, int64_t *shape, int *ndim) {
  if (!a) return fail("shape: null array");
  for (int i = 0; i < a->ndim; i++) shape[i] = a->shape[i];
  *ndim = a->ndim;
  return 0;
}

int shlo_dtype(shlo_arr a, uint8_t *dtype) {
  if (!a) return fail("dtype: null array");
  *dtype = a->dtype;
  return 0;
}

// Strides that read a strided array in a new shape without a copy, when its
// dimensions merge and split only across runs of dimensions that are laid out
// row-contiguously among themselves (size-1 dimensions ignored); false when
// the new shape needs a copy.
static bool reshape_strides(const Arr *a, const int64_t *shape, int ndim, int64_t *st) {
  int64_t od[kMaxRank], os[kMaxRank];
  int on = 0;
  for (int i = 0; i < a->ndim; i++)
    if (a->shape[i] != 1) {
      od[on] = a->shape[i];
      os[on] = a->strides[i];
      on++;
    }
  int oi = 0, ni = 0;
  for (int i = 0; i < ndim; i++) st[i] = 1;
  while (ni < ndim && oi < on) {
    if (shape[ni] == 1) {
      ni++;
      continue;
    }
    int oj = oi + 1, nj = ni + 1;
    int64_t np = shape[ni], op = od[oi];
    while (np != op) {
      if (np < op) {
        if (nj >= ndim) return false;
        np *= shape[nj++];
      } else {
        if (oj >= on) return false;
        op *= od[oj++];
      }
    }
    for (int k = oi; k < oj - 1; k++)
      if (os[k] != od[k + 1] * os[k + 1]) return false;
    st[nj - 1] = os[oj - 1];
    for (int k = nj - 1; k > ni; k--) st[k - 1] = st[k] * shape[k];
    ni = nj;
    oi = oj;
  }
  return oi == on;
}

int shlo_reshape(shlo_arr a, const int64_t *shape, int ndim, shlo_arr *out) {
  if (!a) return fail("reshape: null array");
  if (ndim > kMaxRank) return fail("reshape: rank above %d", kMaxRank);
  int64_t n = 1;
  for (int i = 0; i < ndim; i++) {
    if (shape[i] < 0) return fail("reshape: negative dimension");
    n *= shape[i];
  }
  if (n != numel(a)) return fail("reshape: %lld elements into %lld", (long long)numel(a), (long long)n);
  int64_t st[kMaxRank];
  if (!is_row_contiguous(a) && n > 0 && reshape_strides(a, shape, ndim, st)) {
    // The same storage read with new strides: no copy.
    Arr *v = new_view(a);
    v->ndim = ndim;
    for (int i = 0; i < ndim; i++) {
      v->shape[i] = shape[i];
      v->strides[i] = st[i];
    }
    *out = v;
    return 0;
  }
  // A row-contiguous array keeps its storage; any other is copied first (a
  // read of its data: logged while a compiled function is recorded).
  const bool copies = !is_row_contiguous(a) && a->buf;
  TraceScope ts(copies ? TK_COPY : 0, 1, nullptr, 0, &a, copies ? 1 : 0);
  if (copies && ts.substituted()) return ts.take(out);
  Arr *c;
  SHLO_TRY(make_contiguous(a, &c));
  Arr *v = new_view(c);
  v->ndim = ndim;
  for (int i = 0; i < ndim; i++) v->shape[i] = shape[i];
  set_row_major(v);
  if (c->has_host) {
    v->host = c->host;
    v->has_host = true;
  }
  release_arr(c);
  *out = v;
  if (copies) ts.done(v);
  return 0;
}

int shlo_transpose(shlo_arr a, const int64_t *perm, int ndim, shlo_arr *out) {
  if (!a) return fail("transpose: null array");
  if (ndim != a->ndim) return fail("transpose: %d axes for a rank-%d array", ndim, a->ndim);
  bool seen[kMaxRank] = {false};
  for (int i = 0; i < ndim; i++) {
    if (perm[i] < 0 || perm[i] >= ndim || seen[perm[i]]) return fail("transpose: not a permutation");
    seen[perm[i]] = true;
  }
  Arr *v = new_view(a);
  for (int i = 0; i < ndim; i++) {
    v->shape[i] = a->shape[perm[i]];
    v->strides[i] = a->strides[perm[i]];
  }
  *out = v;
  return 0;
}

int shlo_broadcast(shlo_arr a, const int64_t *shape, int ndim, shlo_arr *out) {
  if (!a) return fail("broadcast: null array");
  return broadcast_view(a, shape, ndim, out);
}

int shlo_slice(shlo_arr a, const int64_t *start, const int64_t *stop, const int64_t *step, int n,
               shlo_arr *out) {
  if (!a) return fail("slice: null array");
  if (n != a->ndim) return fail("slice: %d axes for a rank-%d array", n, a->ndim);
  Arr *v = new_view(a);
  for (int i = 0; i < n; i++) {
    int64_t d = a->shape[i];
    int64_t s = start[i], e = stop[i], k = step[i];
    if (k <= 0) {
      release_arr(v);
      return fail("slice: step %lld on axis %d not carried", (long long)k, i);
    }
    if (s < 0) s += d;
    if (e < 0) e += d;
    s = s < 0 ? 0 : (s > d ? d : s);
    e = e < 0 ? 0 : (e > d ? d : e);
    int64_t len = e > s ? (e - s + k - 1) / k : 0;
    v->offset += s * a->strides[i];
    v->shape[i] = len;
    v->strides[i] = a->strides[i] * k;
  }
  *out = v;
  return 0;
}

int shlo_view(shlo_arr a, uint8_t dtype, shlo_arr *out) {
  if (!a) return fail("view: null array");
  if (!dtype_valid(dtype)) return fail("view: dtype %d not carried", (int)dtype);
  size_t from = dtype_size(a->dtype), to = dtype_size(dtype);
  if (from == to) {
    Arr *v = new_view(a);
    v->dtype = dtype;
    if (a->has_host) {
      v->host = a->host;
      v->has_host = true;
    }
    *out = v;
    return 0;
  }
  if (a->ndim == 0) return fail("view: a scalar cannot change its element size");
  int64_t last = a->shape[a->ndim - 1] * (int64_t)from;
  if (last % (int64_t)to) return fail("view: last axis of %lld bytes is not a multiple of %zu", (long long)last, to);
  TraceScope ts(TK_OTHER, 22, nullptr, 0, &a, 1);  // may copy: logged as a read
  ts.done(nullptr);
  Arr *c;
  SHLO_TRY(make_contiguous(a, &c));
  Arr *v = new_view(c);
  v->dtype = dtype;
  v->shape[v->ndim - 1] = last / (int64_t)to;
  set_row_major(v);
  if ((c->offset * (int64_t)from) % (int64_t)to) {
    release_arr(v);
    release_arr(c);
    return fail("view: misaligned offset");
  }
  v->offset = c->offset * (int64_t)from / (int64_t)to;
  release_arr(c);
  *out = v;
  return 0;
}

int shlo_contiguous(shlo_arr a, shlo_arr *out) {
  if (!a) return fail("contiguous: null array");
  const bool copies = !is_row_contiguous(a) && a->buf;
  TraceScope ts(copies ? TK_COPY : 0, 2, nullptr, 0, &a, copies ? 1 : 0);
  if (copies && ts.substituted()) return ts.take(out);
  const int rc = make_contiguous(a, out);
  if (copies && !rc) ts.done(*out);
  return rc;
}

int shlo_eval(const shlo_arr *xs, int n) {
  bool done[64] = {false};
  for (int i = 0; i < n; i++) {
    if (!xs[i] || !xs[i]->buf) continue;
    int id = xs[i]->buf->dev->id;
    if (done[id]) continue;
    done[id] = true;
    Device *dev;
    SHLO_TRY(device_by_id(id, &dev));
    SHLO_TRY(wait_device(dev, "eval"));
  }
  if (n == 0) {
    Device *dev;
    SHLO_TRY(current_device(&dev));
    SHLO_TRY(wait_device(dev, "eval"));
  }
  return 0;
}

}  // extern "C"
