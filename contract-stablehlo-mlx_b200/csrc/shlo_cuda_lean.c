/*
 * The Lean side of the boundary: the 25 `smlx_*` symbols that
 * StablehloMlx/Mlx.lean:16-73 declares with @[extern], over the plain C ABI of
 * include/shlo_cuda.h. This file takes the place of the reference's
 * c/smlx_shim.c in the Lean build (lakefile.lean:23-31); it unpacks Lean
 * objects, makes one shlo_* call, and boxes the result -- no numerics here.
 *
 * Build (where Lean 4 is installed): compile with the Lean include path and
 * link against libshlo_cuda.so, e.g.
 *   cc -O2 -fPIC -I$(lean --print-prefix)/include -Iinclude -c shlo_cuda_lean.c
 */
#include <lean/lean.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "../../include/shlo_cuda.h"

/* Lean runtime functions this file calls that lean.h does not declare. */
extern lean_object *lean_io_error_to_string(lean_object *err);

/* An IO error whose text is `msg`. */
static lean_obj_res fail_with(const char *msg) {
	return lean_io_result_mk_error(lean_mk_io_user_error(lean_mk_string(msg)));
}

/* A library call failed: the text names the operation and carries the
   library's message for this thread. */
static lean_obj_res lib_error(const char *op) {
	const char *why = shlo_last_error();
	size_t n = strlen(op) + strlen(why) + 3;
	char *msg = (char *)malloc(n);
	if (!msg) return fail_with(op);
	memcpy(msg, op, strlen(op));
	memcpy(msg + strlen(op), ": ", 2);
	memcpy(msg + strlen(op) + 2, why, strlen(why) + 1);
	lean_obj_res r = fail_with(msg);
	free(msg);
	return r;
}

/* ---- external classes: Arr, Kernel, Fn ---- */

static void noop_foreach(void *p, b_lean_obj_arg f) { (void)p; (void)f; }
static void arr_finalize(void *p) { shlo_release((shlo_arr)p); }
static void kern_finalize(void *p) { shlo_kernel_free((shlo_kernel)p); }
static void fn_finalize(void *p) { shlo_fn_free((shlo_fn)p); }
static lean_external_class *arr_class, *kern_class, *fn_class;

static lean_object *box_arr(shlo_arr a) {
	if (!arr_class) arr_class = lean_register_external_class(arr_finalize, noop_foreach);
	return lean_alloc_external(arr_class, a);
}
static shlo_arr unbox_arr(b_lean_obj_arg o) { return (shlo_arr)lean_get_external_data(o); }

/* The entries of an `Array Nat` (a shape, permutation, start/stop/step or a
   grid) as int64 values; false when there are more than `cap`. */
static int read_dims(b_lean_obj_arg dims, int64_t *out, int cap, int *count) {
	size_t len = lean_array_size(dims);
	if (len > (size_t)cap) return 0;
	for (size_t k = 0; k < len; k++) {
		size_t v = lean_unbox(lean_array_get_core(dims, k));
		out[k] = (int64_t)v;
	}
	*count = (int)len;
	return 1;
}

static lean_obj_res ok_arr(int rc, shlo_arr r, const char *what) {
	if (rc) return lib_error(what);
	return lean_io_result_mk_ok(box_arr(r));
}

static lean_object *shape_to_lean(const int64_t *s, int n) {
	lean_object *r = lean_alloc_array(0, (size_t)n);
	for (int i = 0; i < n; i++) r = lean_array_push(r, lean_box((size_t)s[i]));
	return r;
}

/* ---- construction and readback (Mlx.lean:16, 39-42) ---- */

LEAN_EXPORT lean_obj_res smlx_empty(lean_obj_arg u) {
	(void)u;
	return box_arr(shlo_empty());
}

LEAN_EXPORT lean_obj_res smlx_of_bytes(b_lean_obj_arg data, b_lean_obj_arg shape, uint8_t dt, lean_obj_arg w) {
	(void)w;
	int64_t s[SHLO_MAX_RANK];
	int n = 0;
	if (!read_dims(shape, s, SHLO_MAX_RANK, &n)) return fail_with("ofBytes: a shape of more than 16 dimensions");
	shlo_arr r = NULL;
	int rc = shlo_of_bytes(lean_sarray_cptr(data), lean_sarray_size(data), s, n, dt, &r);
	return ok_arr(rc, r, "ofBytes");
}

LEAN_EXPORT lean_obj_res smlx_to_bytes(b_lean_obj_arg a, lean_obj_arg w) {
	(void)w;
	size_t bytes = 0;
	if (shlo_nbytes(unbox_arr(a), &bytes)) return lib_error("toBytes");
	lean_object *r = lean_alloc_sarray(1, bytes, bytes);
	if (shlo_to_bytes(unbox_arr(a), lean_sarray_cptr(r), bytes)) {
		lean_dec(r);
		return lib_error("toBytes");
	}
	return lean_io_result_mk_ok(r);
}

LEAN_EXPORT lean_obj_res smlx_shape(b_lean_obj_arg a, lean_obj_arg w) {
	(void)w;
	int64_t s[SHLO_MAX_RANK];
	int n = 0;
	if (shlo_shape(unbox_arr(a), s, &n)) return lib_error("shape");
	return lean_io_result_mk_ok(shape_to_lean(s, n));
}

LEAN_EXPORT lean_obj_res smlx_dtype(b_lean_obj_arg a, lean_obj_arg w) {
	(void)w;
	uint8_t d = 0;
	if (shlo_dtype(unbox_arr(a), &d)) return lib_error("dtype");
	return lean_io_result_mk_ok(lean_box((size_t)d));
}

/* ---- ops (Mlx.lean:44-58) ---- */

LEAN_EXPORT lean_obj_res smlx_unary(uint32_t op, b_lean_obj_arg a, lean_obj_arg w) {
	(void)w;
	shlo_arr r = NULL;
	return ok_arr(shlo_unary(op, unbox_arr(a), &r), r, "unary");
}

LEAN_EXPORT lean_obj_res smlx_binary(uint32_t op, b_lean_obj_arg a, b_lean_obj_arg b, lean_obj_arg w) {
	(void)w;
	shlo_arr r = NULL;
	return ok_arr(shlo_binary(op, unbox_arr(a), unbox_arr(b), &r), r, "binary");
}

LEAN_EXPORT lean_obj_res smlx_where(b_lean_obj_arg c, b_lean_obj_arg a, b_lean_obj_arg b, lean_obj_arg w) {
	(void)w;
	shlo_arr r = NULL;
	return ok_arr(shlo_where(unbox_arr(c), unbox_arr(a), unbox_arr(b), &r), r, "where");
}

#define SHAPE_OP(NAME, CALL, WHAT)                                                   \
	LEAN_EXPORT lean_obj_res NAME(b_lean_obj_arg a, b_lean_obj_arg shape, lean_obj_arg w) { \
		(void)w;                                                                     \
		int64_t s[SHLO_MAX_RANK];                                                    \
		int n = 0;                                                                   \
		if (!read_dims(shape, s, SHLO_MAX_RANK, &n))                                 \
			return fail_with(WHAT ": more than 16 dimensions");                      \
		shlo_arr r = NULL;                                                           \
		return ok_arr(CALL(unbox_arr(a), s, n, &r), r, WHAT);                        \
	}
SHAPE_OP(smlx_reshape, shlo_reshape, "reshape")
SHAPE_OP(smlx_transpose, shlo_transpose, "transpose")
SHAPE_OP(smlx_broadcast, shlo_broadcast, "broadcast")

LEAN_EXPORT lean_obj_res smlx_slice(b_lean_obj_arg a, b_lean_obj_arg start, b_lean_obj_arg stop, b_lean_obj_arg step,
                                    lean_obj_arg w) {
	(void)w;
	int64_t s0[SHLO_MAX_RANK], s1[SHLO_MAX_RANK], s2[SHLO_MAX_RANK];
	int n = 0, m = 0, k = 0;
	if (!read_dims(start, s0, SHLO_MAX_RANK, &n) || !read_dims(stop, s1, SHLO_MAX_RANK, &m) ||
	    !read_dims(step, s2, SHLO_MAX_RANK, &k) || n != m || n != k)
		return fail_with("slice: start, stop and step must have one entry per dimension (at most 16)");
	shlo_arr r = NULL;
	return ok_arr(shlo_slice(unbox_arr(a), s0, s1, s2, n, &r), r, "slice");
}

LEAN_EXPORT lean_obj_res smlx_concat(b_lean_obj_arg xs, uint32_t axis, lean_obj_arg w) {
	(void)w;
	size_t n = lean_array_size(xs);
	shlo_arr *v = (shlo_arr *)malloc(sizeof(shlo_arr) * (n ? n : 1));
	for (size_t i = 0; i < n; i++) v[i] = unbox_arr(lean_array_get_core(xs, i));
	shlo_arr r = NULL;
	int rc = shlo_concat(v, (int)n, axis, &r);
	free(v);
	return ok_arr(rc, r, "concatenate");
}

LEAN_EXPORT lean_obj_res smlx_astype(b_lean_obj_arg a, uint8_t dt, lean_obj_arg w) {
	(void)w;
	shlo_arr r = NULL;
	return ok_arr(shlo_astype(unbox_arr(a), dt, &r), r, "astype");
}

LEAN_EXPORT lean_obj_res smlx_view(b_lean_obj_arg a, uint8_t dt, lean_obj_arg w) {
	(void)w;
	shlo_arr r = NULL;
	return ok_arr(shlo_view(unbox_arr(a), dt, &r), r, "view");
}

LEAN_EXPORT lean_obj_res smlx_take(b_lean_obj_arg a, b_lean_obj_arg idx, uint32_t axis, lean_obj_arg w) {
	(void)w;
	shlo_arr r = NULL;
	return ok_arr(shlo_take(unbox_arr(a), unbox_arr(idx), axis, &r), r, "take");
}

LEAN_EXPORT lean_obj_res smlx_max_axis(b_lean_obj_arg a, uint32_t axis, lean_obj_arg w) {
	(void)w;
	shlo_arr r = NULL;
	return ok_arr(shlo_max_axis(unbox_arr(a), axis, &r), r, "max_axis");
}

LEAN_EXPORT lean_obj_res smlx_contiguous(b_lean_obj_arg a, lean_obj_arg w) {
	(void)w;
	shlo_arr r = NULL;
	return ok_arr(shlo_contiguous(unbox_arr(a), &r), r, "contiguous");
}

LEAN_EXPORT lean_obj_res smlx_eval(b_lean_obj_arg xs, lean_obj_arg w) {
	(void)w;
	size_t n = lean_array_size(xs);
	shlo_arr *v = (shlo_arr *)malloc(sizeof(shlo_arr) * (n ? n : 1));
	for (size_t i = 0; i < n; i++) v[i] = unbox_arr(lean_array_get_core(xs, i));
	int rc = shlo_eval(v, (int)n);
	free(v);
	if (rc) return lib_error("eval");
	return lean_io_result_mk_ok(lean_box(0));
}

/* ---- kernels (Mlx.lean:60-64) ---- */

LEAN_EXPORT lean_obj_res smlx_kernel_new(b_lean_obj_arg name, b_lean_obj_arg ins, b_lean_obj_arg outs,
                                         b_lean_obj_arg src, b_lean_obj_arg hdr, lean_obj_arg w) {
	(void)w;
	if (!kern_class) kern_class = lean_register_external_class(kern_finalize, noop_foreach);
	size_t ni = lean_array_size(ins), no = lean_array_size(outs);
	const char **vi = (const char **)malloc(sizeof(char *) * (ni ? ni : 1));
	const char **vo = (const char **)malloc(sizeof(char *) * (no ? no : 1));
	for (size_t i = 0; i < ni; i++) vi[i] = lean_string_cstr(lean_array_get_core(ins, i));
	for (size_t i = 0; i < no; i++) vo[i] = lean_string_cstr(lean_array_get_core(outs, i));
	shlo_kernel k = NULL;
	int rc = shlo_kernel_new(lean_string_cstr(name), vi, (int)ni, vo, (int)no, lean_string_cstr(src),
	                         lean_string_cstr(hdr), &k);
	free(vi);
	free(vo);
	if (rc) return lib_error("kernel");
	return lean_io_result_mk_ok(lean_alloc_external(kern_class, k));
}

LEAN_EXPORT lean_obj_res smlx_kernel_apply(b_lean_obj_arg ko, b_lean_obj_arg ins, b_lean_obj_arg shapes,
                                           b_lean_obj_arg dts, b_lean_obj_arg grid, b_lean_obj_arg tg, lean_obj_arg w) {
	(void)w;
	size_t ni = lean_array_size(ins), no = lean_array_size(shapes);
	if (no > 8) return fail_with("kernelApply: more than 8 outputs");
	if (lean_sarray_size(dts) < no) return fail_with("kernelApply: fewer output dtypes than output shapes");
	shlo_arr *vi = (shlo_arr *)malloc(sizeof(shlo_arr) * (ni ? ni : 1));
	for (size_t i = 0; i < ni; i++) vi[i] = unbox_arr(lean_array_get_core(ins, i));
	int64_t sh[8][SHLO_MAX_RANK];
	const int64_t *shp[8];
	int nd[8];
	for (size_t i = 0; i < no; i++) {
		shp[i] = sh[i];
		if (!read_dims(lean_array_get_core(shapes, i), sh[i], SHLO_MAX_RANK, &nd[i])) {
			free(vi);
			return fail_with("kernelApply: an output shape of more than 16 dimensions");
		}
	}
	int64_t g[3], t[3];
	int ng = 0, nt = 0;
	if (!read_dims(grid, g, 3, &ng) || !read_dims(tg, t, 3, &nt) || ng != 3 || nt != 3) {
		free(vi);
		return fail_with("kernelApply: the grid and the threadgroup are [x, y, z] triples");
	}
	shlo_arr outs[8] = {0};
	int rc = shlo_kernel_apply((shlo_kernel)lean_get_external_data(ko), vi, (int)ni, shp, nd, lean_sarray_cptr(dts),
	                           (int)no, g, t, outs);
	free(vi);
	if (rc) return lib_error("kernel apply");
	lean_object *r = lean_alloc_array(0, no);
	for (size_t i = 0; i < no; i++) r = lean_array_push(r, box_arr(outs[i]));
	return lean_io_result_mk_ok(r);
}

/* ---- traced functions (Mlx.lean:66-67) ---- */

/* Calls the Lean closure (Array Arr -> IO (Array Arr)) on the inputs; its error
   message travels back through `err` (c/smlx_shim.c:337-357). */
static int trampoline(void *payload, const shlo_arr *ins, int nin, shlo_arr *outs, int *nout, int max_out, char *err,
                      size_t cap) {
	lean_object *f = (lean_object *)payload;
	lean_object *args = lean_alloc_array(0, (size_t)nin);
	for (int i = 0; i < nin; i++) {
		shlo_retain(ins[i]);
		args = lean_array_push(args, box_arr(ins[i]));
	}
	lean_inc(f);
	lean_object *r = lean_apply_2(f, args, lean_io_mk_world());
	if (lean_io_result_is_error(r)) {
		lean_object *e = lean_io_result_get_error(r);
		lean_inc(e);
		lean_object *msg = lean_io_error_to_string(e);
		snprintf(err, cap, "%s", lean_string_cstr(msg));
		lean_dec(msg);
		lean_dec(r);
		return 1;
	}
	lean_object *res = lean_io_result_get_value(r);
	size_t n = lean_array_size(res);
	if ((int)n > max_out) {
		snprintf(err, cap, "%zu outputs, room for %d", n, max_out);
		lean_dec(r);
		return 1;
	}
	for (size_t i = 0; i < n; i++) {
		shlo_arr a = unbox_arr(lean_array_get_core(res, i));
		shlo_retain(a);
		outs[i] = a;
	}
	*nout = (int)n;
	lean_dec(r);
	return 0;
}

static void payload_free(void *p) { lean_dec((lean_object *)p); }

LEAN_EXPORT lean_obj_res smlx_compile(lean_obj_arg f, uint8_t enable, lean_obj_arg w) {
	(void)w;
	if (!fn_class) fn_class = lean_register_external_class(fn_finalize, noop_foreach);
	shlo_fn fn = NULL;
	if (shlo_compile(trampoline, f, payload_free, enable, &fn)) {
		lean_dec(f);
		return lib_error("compile");
	}
	return lean_io_result_mk_ok(lean_alloc_external(fn_class, fn));
}

LEAN_EXPORT lean_obj_res smlx_apply(b_lean_obj_arg fo, b_lean_obj_arg ins, lean_obj_arg w) {
	(void)w;
	size_t ni = lean_array_size(ins);
	shlo_arr *vi = (shlo_arr *)malloc(sizeof(shlo_arr) * (ni ? ni : 1));
	for (size_t i = 0; i < ni; i++) vi[i] = unbox_arr(lean_array_get_core(ins, i));
	shlo_arr outs[64];
	int n = 0;
	int rc = shlo_apply((shlo_fn)lean_get_external_data(fo), vi, (int)ni, outs, &n, 64);
	free(vi);
	if (rc) return lib_error("apply");
	lean_object *r = lean_alloc_array(0, (size_t)n);
	for (int i = 0; i < n; i++) r = lean_array_push(r, box_arr(outs[i]));
	return lean_io_result_mk_ok(r);
}

/* ---- test-driver helpers (Mlx.lean:69-73) ---- */

LEAN_EXPORT lean_obj_res smlx_libm_erff_range(uint32_t base, uint32_t count, lean_obj_arg w) {
	(void)w;
	lean_object *r = lean_alloc_sarray(1, (size_t)count * 4, (size_t)count * 4);
	if (shlo_libm_erff_range(base, count, (uint32_t *)lean_sarray_cptr(r))) {
		lean_dec(r);
		return lib_error("libm_erff_range");
	}
	return lean_io_result_mk_ok(r);
}

LEAN_EXPORT lean_obj_res smlx_count_nonzero(b_lean_obj_arg a, lean_obj_arg w) {
	(void)w;
	uint64_t n = 0;
	if (shlo_count_nonzero(unbox_arr(a), &n)) return lib_error("count_nonzero");
	return lean_io_result_mk_ok(lean_uint64_to_nat(n));
}
