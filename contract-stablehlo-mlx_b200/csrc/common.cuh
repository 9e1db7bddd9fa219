// Internal declarations shared by the shlo_cuda translation units.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/shlo_cuda.h"

namespace shlo {

constexpr int kMaxRank = SHLO_MAX_RANK;

// ---- dtypes (mlx-c codes, StablehloMlx/Mlx.lean:30-37) ----
enum DType : uint8_t {
  kBool = 0, kU8 = 1, kU16 = 2, kU32 = 3, kU64 = 4,
  kI8 = 5, kI16 = 6, kI32 = 7, kI64 = 8, kF16 = 9, kF32 = 10, kNumDTypes = 11
};
bool dtype_valid(int dt);
size_t dtype_size(int dt);
const char *dtype_name(int dt);
bool dtype_is_float(int dt);
bool dtype_is_signed_int(int dt);
bool dtype_is_unsigned_int(int dt);
int promote_types(int a, int b);

// ---- errors ----
// Record an error message for this host thread and return 1.
int fail(const char *fmt, ...);
// Check a CUDA call; on error record it and return 1.
int cuda_check(cudaError_t e, const char *what);
#define SHLO_CUDA(call)                                \
  do {                                                 \
    if (::shlo::cuda_check((call), #call)) return 1;   \
  } while (0)
#define SHLO_TRY(call)                                 \
  do {                                                 \
    if ((call) != 0) return 1;                         \
  } while (0)

// ---- per-device state ----
struct Device {
  int id = 0;
  int sm_count = 0;
  cudaStream_t stream = nullptr;  // all compute
  cudaStream_t copy = nullptr;    // device-to-host copies of shlo_to_bytes
  std::mutex mu;                  // allocator
  std::multimap<size_t, void *> free_blocks;
  size_t pooled_bytes = 0;
  // Blocks of shlo_of_bytes's uploads, each with the event recorded on `stream`
  // when it was released (see alloc_upload).
  std::multimap<size_t, std::pair<void *, cudaEvent_t>> upload_free;
  // A CUDA-graph capture in progress on `stream` (shlo_apply of a compiled
  // function): blocks allocated meanwhile belong to `capture_owner` and are
  // listed in `capture_allocs`; blocks the capture frees go to `capture_free`
  // and are reused only by later allocations of the same capture (the graph is
  // one linear chain of nodes, so stream order makes that reuse safe).
  // Set by a kernel that gave up a bounded wait (mul_mat's stage pipeline): a
  // word of mapped pinned host memory, read after the device's stream drains.
  int *pipe_err_host = nullptr;
  int *pipe_err_dev = nullptr;
  bool capturing = false;
  void *capture_owner = nullptr;
  std::vector<std::pair<void *, size_t>> *capture_allocs = nullptr;
  std::multimap<size_t, void *> capture_free;
};
// The device current on this host thread, initialised on first use.
int current_device(Device **out);
int device_by_id(int id, Device **out);
int current_flavor();

// ---- storage ----
struct Buffer {
  std::atomic<int> rc{1};
  uint64_t serial = 0;  // unique per storage block made (the op log's identity of data)
  Device *dev = nullptr;
  void *ptr = nullptr;
  size_t bytes = 0;
  // The captured graph this block belongs to (nullptr: the pool's). Such a
  // block is never pooled while the graph lives.
  void *graph_owner = nullptr;
  bool no_recycle = false;  // written at capture time (a constant): never reused inside the capture
  // Recorded on the compute stream right after the buffer was written, where a
  // reader off that stream may come (the results of a graph replay): the
  // device-to-host copy of shlo_to_bytes waits for it and nothing later.
  cudaEvent_t ready = nullptr;
  bool upload = false;  // from the upload pool (shlo_of_bytes on the copy stream)
  // Derived layouts (e.g. the packed operand of mul_mat), keyed by how they
  // were derived, each with the launch that derives it again. Storage is
  // immutable once written, so they stay valid for the buffer's lifetime; the
  // one exception is the private input copy of a compiled function, which is
  // rewritten between replays and then re-derives them (buffer_rederive).
  std::mutex derived_mu;
  std::map<std::string, Buffer *> derived;
  std::map<std::string, std::function<int()>> rederive;
};
int buffer_alloc(Device *dev, size_t bytes, Buffer **out);
// A block for data written by the host at capture time (see shlo_of_bytes).
int buffer_alloc_constant(Device *dev, size_t bytes, Buffer **out);
int buffer_rederive(Buffer *b);
void buffer_retain(Buffer *b);
void buffer_release(Buffer *b);

}  // namespace shlo

// The array handle (opaque in the C ABI).
struct shlo_arr_s {
  std::atomic<int> rc{1};
  uint8_t dtype = shlo::kF32;
  int ndim = 0;
  int64_t shape[shlo::kMaxRank] = {0};
  int64_t strides[shlo::kMaxRank] = {0};  // in elements
  int64_t offset = 0;                     // in elements
  shlo::Buffer *buf = nullptr;            // nullptr for the empty array
  // Host copy of small arrays made by shlo_of_bytes (row-major): the kernel
  // parameter words are read from here without a device round trip.
  std::vector<uint8_t> host;
  bool has_host = false;
};

namespace shlo {

using Arr = shlo_arr_s;

int64_t numel(const Arr *a);
bool is_row_contiguous(const Arr *a);
void set_row_major(Arr *a);
// A new array of `shape` with fresh row-major storage on device `dev`.
int new_array(Device *dev, uint8_t dtype, const int64_t *shape, int ndim, Arr **out);
// A new handle sharing `src`'s storage (the caller sets shape/strides/offset).
Arr *new_view(const Arr *src);
int arr_device(const Arr *a, Device **out);
// A row-contiguous version of `a` (a new reference to `a` itself when it already is).
int make_contiguous(Arr *a, Arr **out);
// Element pointer of the array's first element.
inline char *data_ptr(const Arr *a) {
  return a->buf ? static_cast<char *>(a->buf->ptr) + a->offset * (int64_t)dtype_size(a->dtype) : nullptr;
}
// Read `n` 32-bit words of a small array (host copy, or a synchronous readback).
int read_words(Arr *a, uint32_t *words, int n);

// ---- strided iteration descriptors passed by value to kernels ----
struct StridedDesc {
  int ndim;
  int64_t shape[kMaxRank];
  int64_t strides[kMaxRank];  // per operand, set by the op
};

// Copy `src` (any strides) into the contiguous buffer `dst` (same dtype).
int launch_copy_strided(Device *dev, const Arr *src, void *dst);
// Broadcast `a` to `shape` (stride-0 view) -- no copy.
int broadcast_view(Arr *a, const int64_t *shape, int ndim, Arr **out);
// numpy broadcast of two shapes.
int broadcast_shapes(const int64_t *a, int na, const int64_t *b, int nb, int64_t *out, int *nout);
int cast_array(Arr *a, uint8_t dtype, Arr **out);

// Kernel launch size helper: a grid-stride launch over n elements.
inline unsigned grid_for(int64_t n, int threads, Device *dev, int per_sm = 8) {
  int64_t blocks = (n + threads - 1) / threads;
  int64_t cap = (int64_t)dev->sm_count * per_sm;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return (unsigned)blocks;
}

inline float bitsf_host(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

// Launch-error check after a kernel launch.
int launch_check(const char *what);
// Kernel launches made through launch_check since the library was loaded.
extern std::atomic<uint64_t> g_launches;
// Wait for all queued work of a device (bounded by SHLO_EVAL_TIMEOUT_S).
int device_wait(Device *dev, const char *what);

// The kernels of shlo_kernel_apply, by name (api.cu's table).
enum KernelKind {
  KK_MUL_MAT, KK_SOFT_MAX, KK_NORM, KK_SILU, KK_GELU_ERF, KK_ERFF_MAP, KK_DIVIDE, KK_SQRT, KK_F64_EW,
  KK_F64_OF_F32, KK_F32_OF_F64, KK_MUL_MAT_EP, KK_NORM_AFFINE, KK_ATTENTION
};
// mul_mat's fused epilogue (k_mul_mat_ep): + bias[m] (its own operand order),
// then + res[r][m], then gelu_erf (the pinned build's).
enum { EP_BIAS = 1, EP_BIAS_LHS = 2, EP_RES = 4, EP_RES_LHS = 8, EP_GELU = 16 };

// ---- recording a compiled function: the op log and its fusions (fusion.cu) ----
// Entry points that read array data open a TraceScope. While the recorder logs
// the eager call of a compiled function (shlo_apply's first call of a
// signature), the outermost scope on the thread logs the op; in the capture
// call that follows, an op of a fusable chain is substituted: the scope then
// holds the op's result (a placeholder, or the fused kernel's result at the
// chain's end) and the entry point returns it without running the op.
enum TraceKind { TK_KERNEL = 1, TK_BINARY, TK_COPY, TK_OTHER };
struct Tracer;
extern thread_local Tracer *t_tracer;
bool fusion_enabled();
Tracer *tracer_new(Device *dev);
void tracer_free(Tracer *t);
// After the eager call: mark its outputs, find the chains, switch to the capture
// call's mode. Returns the number of chains found.
int tracer_plan(Tracer *t, shlo_arr_s *const *outs, int n);
// After the capture call: whether it matched the log and ended every chain.
bool tracer_complete(Tracer *t, std::string *why);

class TraceScope {
 public:
  TraceScope(int kind, int sub, const uint32_t *p, int np, shlo_arr_s *const *ins, int n);
  ~TraceScope();
  TraceScope(const TraceScope &) = delete;
  TraceScope &operator=(const TraceScope &) = delete;
  bool substituted() const { return substituted_; }
  // The substituted op's status, with its result in *out on success.
  int take(shlo_arr_s **out) {
    *out = result_;
    return status_;
  }
  // The op ran: log its result (nullptr when it returns no array).
  void done(shlo_arr_s *out);

 private:
  int depth_ = 0, idx_ = -1, status_ = 0;
  bool logging_ = false, substituted_ = false;
  shlo_arr_s *result_ = nullptr;
};

// ---- ggml kernels (ggml_kernels.cu) ----
int k_mul_mat(Device *dev, Arr *w, Arr *x, const uint32_t *p, Arr **out);
// mul_mat with the executor's fused epilogue: + bias[m] and/or + res[r][m]
// (ep: 1 bias, 2 bias is the add's left operand, 4 residual, 8 residual left).
int k_mul_mat_ep(Device *dev, Arr *w, Arr *x, const uint32_t *p, Arr *bias, Arr *res, int ep, Arr **out);
// k_mul_mat_ep for chained dense products (fusion.cu): x_np > 0, x's storage
// is this product's packed x already (mm_packed_x_layout's layout, x_np padded
// rows); y_pack = {segp, Np}: the result is written in the packed layout of a
// next product whose K is this one's M (its logical shape stays [R*M]).
int k_mul_mat_fused(Device *dev, Arr *w, Arr *x, const uint32_t *p, Arr *bias, Arr *res, int ep, int x_np,
                    const int *y_pack, Arr **out);
// The packed x a product of K x M over R rows (one weight) makes: false where
// it packs none or its x needs segment padding or a tail.
bool mm_packed_x_layout(int64_t K, int64_t M, int64_t R, int *segp, int *Np);
int k_soft_max(Device *dev, Arr *x, const uint32_t *p, Arr **out);
int k_norm(Device *dev, Arr *x, const uint32_t *p, Arr **out);
// norm with the executor's fused affine: (y * gamma[c]) + beta[c].
int k_norm_affine(Device *dev, Arr *x, const uint32_t *p, Arr *gamma, Arr *beta, Arr **out);
// k_norm_affine whose result is the packed x (y_pack = {segp, Np}, as
// mm_packed_x_layout gives it) of a product over the normalised rows.
int k_norm_affine_packed(Device *dev, Arr *x, const uint32_t *p, Arr *gamma, Arr *beta, const int *y_pack,
                         Arr **out);
// The executor's fused attention (scores, soft_max, value product): q, k, v
// [B][S][H][64] views, p = [B, S, H, 64, scale bits]; the result is [B][S][H][64].
int k_attention(Device *dev, Arr *q, Arr *k, Arr *v, const uint32_t *p, Arr **out);
// k_attention whose result is the packed x (y_pack = {segp, Np}, as
// mm_packed_x_layout gives it) of a product over the merged heads.
int k_attention_packed(Device *dev, Arr *q, Arr *k, Arr *v, const uint32_t *p, const int *y_pack, Arr **out);
// A row-major rows x K operand copied into the packed x layout y_pack = {segp,
// Np} (K a multiple of 64; the rows past `rows` zero).
int k_pack_x(Device *dev, Arr *src, int64_t rows, int64_t K, const int *y_pack, Arr **out);
int k_silu(Device *dev, Arr *x, const uint32_t *p, Arr **out);
int k_gelu_erf(Device *dev, Arr *x, const uint32_t *p, Arr **out);
int k_erff_map(Device *dev, const uint32_t *p, Arr **out);
int k_divide(Device *dev, Arr *a, Arr *b, const uint32_t *p, Arr **out);
int k_sqrt(Device *dev, Arr *a, const uint32_t *p, Arr **out);
int k_f64_ew(Device *dev, Arr *a, Arr *b, const uint32_t *p, Arr **out);
int k_f64_of_f32(Device *dev, Arr *a, const uint32_t *p, Arr **out);
int k_f32_of_f64(Device *dev, Arr *a, const uint32_t *p, Arr **out);

// ---- built-ins (elementwise.cu) ----
int op_unary(uint32_t op, Arr *a, Arr **out);
int op_binary(uint32_t op, Arr *a, Arr *b, Arr **out);
int op_where(Arr *c, Arr *a, Arr *b, Arr **out);
int op_astype(Arr *a, uint8_t dt, Arr **out);
int op_max_axis(Arr *a, int axis, Arr **out);
int op_count_nonzero(Arr *a, uint64_t *count);
int op_take(Arr *a, Arr *idx, int axis, Arr **out);
int op_concat(Arr *const *xs, int n, int axis, Arr **out);

}  // namespace shlo
