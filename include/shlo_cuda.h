/*
 * shlo_cuda -- a B200 (sm_100a) backend for the StableHLO executor of
 * V-Sekai-fire/contract-stablehlo-mlx, behind the executor's own FFI boundary.
 *
 * The reference binds 25 C symbols from its Lean declarations
 * (StablehloMlx/Mlx.lean:16-73, implemented over mlx-c by c/smlx_shim.c). This
 * header is the same boundary as a plain C ABI: opaque handles, plain pointers
 * and sizes, no Lean or torch types. Each `shlo_*` function below cites the
 * reference declaration it replaces. A thin Lean glue file
 * (contract-stablehlo-mlx_b200/csrc/shlo_cuda_lean.c) exports the exact `smlx_*`
 * symbol names with Lean object conventions on top of it.
 *
 * Conventions
 *  - Every function that can fail returns 0 on success and a nonzero status
 *    otherwise; shlo_last_error() then holds the message (per host thread).
 *    Ops that ggml-cpu computes with code this backend does not carry fail
 *    with a message containing "not carried".
 *  - Arrays are immutable values with reference counts. A function that
 *    returns an array through `shlo_arr *out` hands the caller one reference;
 *    release it with shlo_release(). Views (transpose, broadcast, slice,
 *    reshape of a row-contiguous array) share storage with their source.
 *  - Work is issued asynchronously on one CUDA stream per device; shlo_eval()
 *    waits for it (with a wall-clock limit, SHLO_EVAL_TIMEOUT_S, default 600 s).
 *  - Each host thread has a current device (shlo_set_device); arrays live on
 *    the device that was current when they were made, and an op on arrays of
 *    two devices is an error. Driving each GPU from its own host thread is
 *    supported; one array must not be used from two threads at once.
 *  - dtype codes are mlx-c's (Mlx.lean:30-37): 0 bool, 1 u8, 2 u16, 3 u32,
 *    4 u64, 5 i8, 6 i16, 7 i32, 8 i64, 9 f16, 10 f32.
 */
#ifndef SHLO_CUDA_H
#define SHLO_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SHLO_MAX_RANK 16

typedef struct shlo_arr_s *shlo_arr;       /* Mlx.lean:12-15  `Arr`    */
typedef struct shlo_kernel_s *shlo_kernel; /* Mlx.lean:18-21  `Kernel` */
typedef struct shlo_fn_s *shlo_fn;         /* Mlx.lean:23-26  `Fn`     */

enum shlo_dtype {
	SHLO_BOOL = 0, SHLO_U8 = 1, SHLO_U16 = 2, SHLO_U32 = 3, SHLO_U64 = 4,
	SHLO_I8 = 5, SHLO_I16 = 6, SHLO_I32 = 7, SHLO_I64 = 8, SHLO_F16 = 9, SHLO_F32 = 10
};

/* ---- library state (no counterpart in Mlx.lean; the reference has one GPU) ---- */

/* The last error message of this host thread ("" if none). */
const char *shlo_last_error(void);
/* Select the device for this host thread (default: $SHLO_DEVICE or 0). */
int shlo_set_device(int device);
int shlo_get_device(int *device);
int shlo_device_count(int *count);
/* Which ggml-cpu build the kernels reproduce: 0 = pinned (contract-ggml-stablehlo's
   reference build, the default), 1 = stock (ref/build.sh:10-20). Also read from
   $SHLO_GGML_FLAVOR ("pinned" or "stock") at first use. */
int shlo_set_flavor(int flavor);
int shlo_get_flavor(int *flavor);
/* Take one more reference / drop one (frees the storage at zero). */
void shlo_retain(shlo_arr a);
void shlo_release(shlo_arr a);

/* ---- construction and readback ---- */

/* smlx_empty -- Mlx.lean:16 `emptyArr`: an array with no storage. */
shlo_arr shlo_empty(void);
/* smlx_of_bytes -- Mlx.lean:39 `ofBytes`: copy `nbytes` host bytes (row-major)
   into a new array of `shape` and `dtype`. The bytes are consumed before the
   call returns. nbytes must equal the element count times the dtype size. */
int shlo_of_bytes(const void *data, size_t nbytes, const int64_t *shape, int ndim, uint8_t dtype,
                  shlo_arr *out);
/* smlx_to_bytes -- Mlx.lean:40 `toBytes`: evaluate and copy the array out in
   row-major order. `cap` must be at least shlo_nbytes(a). */
int shlo_nbytes(shlo_arr a, size_t *nbytes);
int shlo_to_bytes(shlo_arr a, void *dst, size_t cap);
/* smlx_shape -- Mlx.lean:41; `shape` has room for SHLO_MAX_RANK entries. */
int shlo_shape(shlo_arr a, int64_t *shape, int *ndim);
/* smlx_dtype -- Mlx.lean:42. */
int shlo_dtype(shlo_arr a, uint8_t *dtype);

/* ---- built-in ops (Mlx.lean:44-58; op codes Mlx.lean:76-108) ---- */

/* smlx_unary: 0 neg, 1 abs, 2 sqrt, 3 floor, 4 exp, 5 erf, 6 logical_not,
   7 bitwise_invert, 8 rsqrt, 9 tanh, 10 sigmoid. */
int shlo_unary(uint32_t op, shlo_arr a, shlo_arr *out);
/* smlx_binary: 0 add, 1 sub, 2 mul, 3 div, 4 max, 5 min, 6 and, 7 or, 8 xor,
   9 shl, 10 shr, 11 eq, 12 ne, 13 lt, 14 le, 15 gt, 16 ge, 17 matmul,
   18 remainder, 19 logical_and, 20 logical_or. Numpy broadcasting and MLX type
   promotion. */
int shlo_binary(uint32_t op, shlo_arr a, shlo_arr b, shlo_arr *out);
/* smlx_where -- Mlx.lean:46. */
int shlo_where(shlo_arr cond, shlo_arr a, shlo_arr b, shlo_arr *out);
/* smlx_reshape -- Mlx.lean:47. */
int shlo_reshape(shlo_arr a, const int64_t *shape, int ndim, shlo_arr *out);
/* smlx_transpose -- Mlx.lean:48 (a permuted view). */
int shlo_transpose(shlo_arr a, const int64_t *perm, int ndim, shlo_arr *out);
/* smlx_broadcast -- Mlx.lean:49 (a stride-0 view). */
int shlo_broadcast(shlo_arr a, const int64_t *shape, int ndim, shlo_arr *out);
/* smlx_slice -- Mlx.lean:50 (start, stop, step per axis; a strided view). */
int shlo_slice(shlo_arr a, const int64_t *start, const int64_t *stop, const int64_t *step, int n,
               shlo_arr *out);
/* smlx_concat -- Mlx.lean:51. */
int shlo_concat(const shlo_arr *xs, int n, uint32_t axis, shlo_arr *out);
/* smlx_astype -- Mlx.lean:52. */
int shlo_astype(shlo_arr a, uint8_t dtype, shlo_arr *out);
/* smlx_view -- Mlx.lean:53 (bit reinterpretation). */
int shlo_view(shlo_arr a, uint8_t dtype, shlo_arr *out);
/* smlx_take -- Mlx.lean:54 (gather along an axis; indices are clamped). */
int shlo_take(shlo_arr a, shlo_arr idx, uint32_t axis, shlo_arr *out);
/* smlx_max_axis -- Mlx.lean:56 (the axis is removed). */
int shlo_max_axis(shlo_arr a, uint32_t axis, shlo_arr *out);
/* smlx_contiguous -- Mlx.lean:57. */
int shlo_contiguous(shlo_arr a, shlo_arr *out);
/* smlx_eval -- Mlx.lean:58: wait until the arrays (all queued work) are computed. */
int shlo_eval(const shlo_arr *xs, int n);

/* ---- custom kernels (Mlx.lean:60-64) ----
   The kernel is chosen by name: "smlx_mul_mat", "smlx_soft_max", "smlx_norm",
   "smlx_silu", "smlx_gelu_erf", "smlx_erff_map", "smlx_divide", "smlx_sqrt",
   "smlx_f64_ew", "smlx_f64_of_f32", "smlx_f32_of_f64" -- the names
   StablehloMlx/Kernels/Run.lean:23 passes. The Metal source and header are
   ignored; any other name is an error. Inputs follow the binding order of
   StablehloMlx/Kernels/Shaders.lean; the parameter words are read from the
   host copy the library keeps of small arrays. Grid and threadgroup are hints
   and are ignored: each kernel chooses its own launch from the parameters. */
int shlo_kernel_new(const char *name, const char *const *inputs, int n_inputs,
                    const char *const *outputs, int n_outputs, const char *source,
                    const char *header, shlo_kernel *out);
void shlo_kernel_free(shlo_kernel k);
int shlo_kernel_apply(shlo_kernel k, const shlo_arr *inputs, int n_inputs,
                      const int64_t *const *out_shapes, const int *out_ndims,
                      const uint8_t *out_dtypes, int n_outputs, const int64_t grid[3],
                      const int64_t threadgroup[3], shlo_arr *outs);

/* ---- traced functions (Mlx.lean:66-67) ----
   `f` computes outputs from inputs by calling this library; it returns 0, or
   nonzero with a message in `err`. With enable = 0 every shlo_apply calls `f`.
   With enable = 1 the first call for each set of input shapes and dtypes is
   captured into a CUDA graph and later calls replay it; the library calls `f`
   again only for a new signature. shlo_compile takes ownership of `payload`
   and calls `payload_free(payload)` when the function is freed. */
typedef int (*shlo_trace_fn)(void *payload, const shlo_arr *inputs, int n_inputs,
                             shlo_arr *outputs, int *n_outputs, int max_outputs,
                             char *err, size_t err_cap);
int shlo_compile(shlo_trace_fn f, void *payload, void (*payload_free)(void *), int enable,
                 shlo_fn *out);
void shlo_fn_free(shlo_fn f);
int shlo_apply(shlo_fn f, const shlo_arr *inputs, int n_inputs, shlo_arr *outputs,
               int *n_outputs, int max_outputs);

/* ---- measurement hooks (no counterpart in the reference: its shim has no timing) ---- */

/* The CUDA stream (a cudaStream_t) on which all work of this thread's current
   device is queued, for timing with CUDA events on the launching stream. */
int shlo_current_stream(void **stream);
/* How many kernels this library has launched since it was loaded, all devices. */
int shlo_launch_count(uint64_t *count);
/* The device address of a row-contiguous array's first element and the device
   it lives on, for handing a result to another library on the same GPU (a
   collective's send buffer, say) without a copy; mlx-c's mlx_array_data_* play
   this part on the reference's unified memory. The array's producing work is
   queued on shlo_current_stream(): order the reader after it (an event on that
   stream), and keep a reference to the array, with the compute stream ordered
   after the reader, until the reader is done -- the storage returns to this
   library's pool when the last reference goes. A strided view is an error. */
int shlo_device_ptr(shlo_arr a, void **ptr, int *device);

/* ---- mul_mat for callers that cannot allocate (no counterpart in the reference) ----
   The same product as the "smlx_mul_mat" kernel (ggml_vec_dot_f32 order, the
   current ggml build; parameters as Run.lean's mulMat: y[r*M+m] = dot of w row
   (r/N)*w_batch_stride + m*K and x row r), for callers whose device memory is
   not this library's to allocate -- a runtime whose GPU memory is all held by
   its own pool or arena, or one that must not allocate while it records work.
   w, x and y are device pointers on the current device (float32, row-major,
   caller-owned); the work is queued on `stream` (a cudaStream_t; NULL is the
   default stream). The packed operands go to one fixed 16 MiB scratch array
   that every GPU loading this library holds until exit; shapes whose packed
   operands need more are rejected with an error. The first call on a device
   looks up the array's address (make it before any stream capture). All calls
   on a device share the array, so calls that overlap on the GPU race: queue
   them on one stream. Nothing is allocated: no cudaMalloc, cudaFree or
   allocating library call. */
int shlo_mul_mat_noalloc(const float *w, const float *x, float *y, int64_t K, int64_t M, int64_t R, int64_t N,
                         int64_t w_batch_stride, void *stream);

/* ---- test-driver helpers (Mlx.lean:69-73) ---- */

/* smlx_libm_erff_range: this platform's binary32 erff over `count`
   consecutive bit patterns from `base`, computed on the host CPU. The
   platform erff of this backend is the correctly rounded one (the pinned
   reference build links CORE-MATH's). `out` receives `count` uint32 words. */
int shlo_libm_erff_range(uint32_t base, uint32_t count, uint32_t *out);
/* smlx_count_nonzero: the exact number of nonzero elements, evaluated. */
int shlo_count_nonzero(shlo_arr a, uint64_t *count);

#ifdef __cplusplus
}
#endif
#endif
