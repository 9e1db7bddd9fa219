/* Runs the Lean glue (contract-stablehlo-mlx_b200/csrc/shlo_cuda_lean.c) the way
 * the Lean executor calls it, over the Lean runtime model (lean_model.c) and
 * libshlo_cuda.so -- test infrastructure only.
 *
 *   lean_glue_run cpu                 checks that need no GPU
 *   lean_glue_run gpu DIR K M R       also the kernel path: DIR/w.f32 ([M,K]) and
 *                                     DIR/x.f32 ([R,K]) in, DIR/out_eager.f32,
 *                                     DIR/out_compiled.f32, DIR/out_replay.f32 out
 *
 * The GPU sequence is Kernels/Run.lean's mulMat as Lower.lean issues it:
 * ofBytes of the operands and of the 8 parameter words, kernelNew
 * "smlx_mul_mat", kernelApply, toBytes; then the same inside a compiled
 * function (Mlx.lean's compile/apply, the closure standing in for
 * Lower.runFunc), applied twice. Then the error paths (a traced function that
 * fails, an unknown kernel, too many outputs, a bad grid) and, once every
 * reference is dropped, that every external object was finalized.
 * Prints one "ok <check>" or "FAIL <check>: <why>" line per check; the exit
 * status is the number of failures.
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <lean/lean.h>

#include "lean_model.h"

/* the glue's exports (StablehloMlx/Mlx.lean:16-73) */
lean_obj_res smlx_empty(lean_obj_arg);
lean_obj_res smlx_of_bytes(b_lean_obj_arg, b_lean_obj_arg, uint8_t, lean_obj_arg);
lean_obj_res smlx_to_bytes(b_lean_obj_arg, lean_obj_arg);
lean_obj_res smlx_shape(b_lean_obj_arg, lean_obj_arg);
lean_obj_res smlx_dtype(b_lean_obj_arg, lean_obj_arg);
lean_obj_res smlx_eval(b_lean_obj_arg, lean_obj_arg);
lean_obj_res smlx_kernel_new(b_lean_obj_arg, b_lean_obj_arg, b_lean_obj_arg, b_lean_obj_arg, b_lean_obj_arg,
                             lean_obj_arg);
lean_obj_res smlx_kernel_apply(b_lean_obj_arg, b_lean_obj_arg, b_lean_obj_arg, b_lean_obj_arg, b_lean_obj_arg,
                               b_lean_obj_arg, lean_obj_arg);
lean_obj_res smlx_compile(lean_obj_arg, uint8_t, lean_obj_arg);
lean_obj_res smlx_apply(b_lean_obj_arg, b_lean_obj_arg, lean_obj_arg);
lean_obj_res smlx_count_nonzero(b_lean_obj_arg, lean_obj_arg);

static int failures;

static void check(int ok, const char *name, const char *why) {
	if (ok)
		printf("ok %s\n", name);
	else {
		printf("FAIL %s: %s\n", name, why ? why : "");
		failures++;
	}
}

/* The value of an ok IO result (one new reference), or NULL after reporting. */
static lean_object *take(lean_object *r, const char *name) {
	if (lean_io_result_is_error(r)) {
		check(0, name, model_error_text(r));
		lean_dec(r);
		return NULL;
	}
	lean_object *v = lean_io_result_get_value(r);
	lean_inc(v);
	lean_dec(r);
	return v;
}

/* The error text of an IO result that must fail, checked for `needle`. */
static void expect_error(lean_object *r, const char *name, const char *needle) {
	const char *msg = model_error_text(r);
	char why[512];
	snprintf(why, sizeof why, "expected an error containing \"%s\", got %s", needle, msg ? msg : "success");
	check(msg && strstr(msg, needle), name, why);
	lean_dec(r);
}

static lean_object *strings(const char **v, int n) {
	lean_object *a = lean_alloc_array(0, (size_t)n);
	for (int i = 0; i < n; i++) a = lean_array_push(a, lean_mk_string(v[i]));
	return a;
}

static lean_object *arr_of(lean_object **v, int n) {
	lean_object *a = lean_alloc_array(0, (size_t)n);
	for (int i = 0; i < n; i++) {
		lean_inc(v[i]);
		a = lean_array_push(a, v[i]);
	}
	return a;
}

static lean_object *kernel(const char *name, int nin) {
	const char *ins[] = {"w", "x", "p"}, *outs[] = {"y"};
	lean_object *nm = lean_mk_string(name), *vi = strings(ins, nin), *vo = strings(outs, 1);
	lean_object *src = lean_mk_string("/* Metal source: ignored by this backend */"), *hdr = lean_mk_string("");
	lean_object *r = smlx_kernel_new(nm, vi, vo, src, hdr, lean_io_mk_world());
	lean_dec(nm);
	lean_dec(vi);
	lean_dec(vo);
	lean_dec(src);
	lean_dec(hdr);
	return r;
}

/* ---- the closures standing in for Lower.runFunc ---- */

struct mm_env {
	lean_object *k, *p;  /* the mul_mat kernel and its parameter words */
	int64_t count;       /* R * M */
};

static lean_object *apply_mm(struct mm_env *e, lean_object *w, lean_object *x) {
	lean_object *ins[3] = {w, x, e->p};
	lean_object *vi = arr_of(ins, 3);
	lean_object *shape = model_nats(&e->count, 1);
	lean_object *shapes = lean_alloc_array(0, 1);
	shapes = lean_array_push(shapes, shape);
	uint8_t f32 = 10;
	lean_object *dts = model_bytes(&f32, 1);
	int64_t g[3] = {e->count, 1, 1}, t[3] = {64, 1, 1};
	lean_object *grid = model_nats(g, 3), *tg = model_nats(t, 3);
	lean_object *r = smlx_kernel_apply(e->k, vi, shapes, dts, grid, tg, lean_io_mk_world());
	lean_dec(vi);
	lean_dec(shapes);
	lean_dec(dts);
	lean_dec(grid);
	lean_dec(tg);
	return r;
}

static lean_object *traced_mm(void *env, lean_object *args, lean_object *world) {
	(void)world;
	lean_object *r = apply_mm((struct mm_env *)env, lean_array_get_core(args, 0), lean_array_get_core(args, 1));
	lean_dec(args);
	return r;
}

static lean_object *traced_fails(void *env, lean_object *args, lean_object *world) {
	(void)env;
	(void)world;
	lean_dec(args);
	return lean_io_result_mk_error(lean_mk_io_user_error(lean_mk_string("composite ggml.rope: not carried")));
}

/* ---- the checks ---- */

static void cpu_checks(void) {
	/* an unknown kernel is refused as not carried */
	expect_error(kernel("smlx_rope", 3), "kernel_new refuses an unknown name", "not carried");

	/* a compiled function whose trace fails: the error comes back through
	   apply with the traced message kept (c/smlx_shim.c:337-357) */
	lean_object *fn = take(smlx_compile(model_closure(traced_fails, NULL), 1, lean_io_mk_world()), "compile");
	if (fn) {
		lean_object *e = smlx_empty(lean_box(0));
		lean_object *ins = arr_of(&e, 1);
		lean_object *r = smlx_apply(fn, ins, lean_io_mk_world());
		const char *msg = model_error_text(r);
		check(msg && strstr(msg, "traced function") && strstr(msg, "ggml.rope: not carried"),
		      "apply returns the traced function's error", msg ? msg : "apply succeeded");
		lean_dec(r);
		lean_dec(ins);
		lean_dec(e);
		lean_dec(fn);
	}

	/* kernelApply with more output shapes than the glue carries, and a grid of
	   two entries: errors, not crashes */
	lean_object *k = take(kernel("smlx_mul_mat", 3), "kernel_new smlx_mul_mat");
	if (k) {
		lean_object *e = smlx_empty(lean_box(0));
		lean_object *ins = arr_of(&e, 1);
		int64_t one = 1;
		lean_object *shapes = lean_alloc_array(0, 9);
		for (int i = 0; i < 9; i++) shapes = lean_array_push(shapes, model_nats(&one, 1));
		uint8_t dts9[9] = {10, 10, 10, 10, 10, 10, 10, 10, 10};
		lean_object *dts = model_bytes(dts9, 9);
		int64_t g[3] = {1, 1, 1};
		lean_object *grid = model_nats(g, 3), *grid2 = model_nats(g, 2);
		expect_error(smlx_kernel_apply(k, ins, shapes, dts, grid, grid, lean_io_mk_world()),
		             "kernel_apply refuses nine outputs", "outputs");
		lean_object *shapes1 = lean_alloc_array(0, 1);
		shapes1 = lean_array_push(shapes1, model_nats(&one, 1));
		expect_error(smlx_kernel_apply(k, ins, shapes1, dts, grid2, grid, lean_io_mk_world()),
		             "kernel_apply refuses a grid of two entries", "grid");
		lean_dec(shapes1);
		lean_dec(grid2);
		lean_dec(grid);
		lean_dec(dts);
		lean_dec(shapes);
		lean_dec(ins);
		lean_dec(e);
		lean_dec(k);
	}
}

static float *read_f32(const char *dir, const char *name, size_t n) {
	char path[1024];
	snprintf(path, sizeof path, "%s/%s", dir, name);
	FILE *f = fopen(path, "rb");
	if (!f) return NULL;
	float *v = (float *)malloc(n * sizeof(float));
	size_t got = fread(v, sizeof(float), n, f);
	fclose(f);
	if (got != n) {
		free(v);
		return NULL;
	}
	return v;
}

static void write_bytes(const char *dir, const char *name, lean_object *bytes) {
	char path[1024];
	snprintf(path, sizeof path, "%s/%s", dir, name);
	FILE *f = fopen(path, "wb");
	if (!f) {
		check(0, name, "cannot write the output file");
		return;
	}
	fwrite(lean_sarray_cptr(bytes), 1, lean_sarray_size(bytes), f);
	fclose(f);
}

static lean_object *of_f32(const float *v, int64_t rows, int64_t cols) {
	lean_object *b = model_bytes(v, (size_t)(rows * cols) * sizeof(float));
	int64_t s[2] = {rows, cols};
	lean_object *shape = model_nats(s, 2);
	lean_object *r = smlx_of_bytes(b, shape, 10, lean_io_mk_world());
	lean_dec(b);
	lean_dec(shape);
	return take(r, "of_bytes");
}

static void gpu_checks(const char *dir, int64_t K, int64_t M, int64_t R) {
	float *w = read_f32(dir, "w.f32", (size_t)(M * K)), *x = read_f32(dir, "x.f32", (size_t)(R * K));
	if (!w || !x) {
		check(0, "inputs", "cannot read w.f32 / x.f32");
		return;
	}
	lean_object *W = of_f32(w, M, K), *X = of_f32(x, R, K);
	free(w);
	free(x);
	uint32_t words[8] = {(uint32_t)K, (uint32_t)M, (uint32_t)R, 0, (uint32_t)R, 0, 0, 0};
	lean_object *pb = model_bytes(words, sizeof words);
	int64_t eight = 8;
	lean_object *ps = model_nats(&eight, 1);
	lean_object *P = take(smlx_of_bytes(pb, ps, 3, lean_io_mk_world()), "of_bytes params");
	lean_dec(pb);
	lean_dec(ps);
	lean_object *k = take(kernel("smlx_mul_mat", 3), "kernel_new smlx_mul_mat");
	if (!W || !X || !P || !k) return;
	struct mm_env env = {k, P, R * M};

	/* eager: kernelApply, then eval and toBytes */
	lean_object *outs = take(apply_mm(&env, W, X), "kernel_apply");
	if (outs) {
		lean_object *y = lean_array_get_core(outs, 0);
		lean_object *ev = arr_of(&y, 1);
		lean_object *ok = take(smlx_eval(ev, lean_io_mk_world()), "eval");
		lean_dec(ok);
		lean_dec(ev);
		lean_object *shape = take(smlx_shape(y, lean_io_mk_world()), "shape");
		check(shape && lean_array_size(shape) == 1 && (int64_t)lean_unbox(lean_array_get_core(shape, 0)) == R * M,
		      "shape of the result", "not [R*M]");
		lean_dec(shape);
		lean_object *dt = take(smlx_dtype(y, lean_io_mk_world()), "dtype");
		check(dt && lean_unbox(dt) == 10, "dtype of the result", "not float32");
		lean_object *nz = take(smlx_count_nonzero(y, lean_io_mk_world()), "count_nonzero");
		check(nz && (int64_t)lean_unbox(nz) > 0, "count_nonzero of the result", "no nonzero word");
		lean_object *bytes = take(smlx_to_bytes(y, lean_io_mk_world()), "to_bytes");
		if (bytes) {
			check(lean_sarray_size(bytes) == (size_t)(R * M) * 4, "to_bytes size", "wrong byte count");
			write_bytes(dir, "out_eager.f32", bytes);
			lean_dec(bytes);
		}
		lean_dec(outs);
	}

	/* compiled: the closure is recorded on the first apply, replayed on the second */
	lean_object *fn = take(smlx_compile(model_closure(traced_mm, &env), 1, lean_io_mk_world()), "compile");
	if (fn) {
		lean_object *two[2] = {W, X};
		const char *files[2] = {"out_compiled.f32", "out_replay.f32"};
		for (int call = 0; call < 2; call++) {
			lean_object *ins = arr_of(two, 2);
			lean_object *res = take(smlx_apply(fn, ins, lean_io_mk_world()), "apply");
			lean_dec(ins);
			if (!res) break;
			check(lean_array_size(res) == 1, "apply returns one array", "wrong count");
			lean_object *bytes = take(smlx_to_bytes(lean_array_get_core(res, 0), lean_io_mk_world()), "to_bytes");
			if (bytes) {
				write_bytes(dir, files[call], bytes);
				lean_dec(bytes);
			}
			lean_dec(res);
		}
		lean_dec(fn);
	}
	lean_dec(k);
	lean_dec(P);
	lean_dec(X);
	lean_dec(W);
}

int main(int argc, char **argv) {
	if (argc < 2) {
		fprintf(stderr, "usage: %s cpu | gpu DIR K M R\n", argv[0]);
		return 2;
	}
	cpu_checks();
	if (strcmp(argv[1], "gpu") == 0) {
		if (argc != 6) {
			fprintf(stderr, "usage: %s gpu DIR K M R\n", argv[0]);
			return 2;
		}
		gpu_checks(argv[2], atoll(argv[3]), atoll(argv[4]), atoll(argv[5]));
	}
	/* every reference dropped: each external object (arrays, kernels,
	   compiled functions) went through its class finalizer */
	char why[128];
	snprintf(why, sizeof why, "%ld made, %ld finalized, %ld objects live", model_externals_made(),
	         model_externals_finalized(), model_objects_live());
	check(model_externals_made() > 0 && model_externals_made() == model_externals_finalized() &&
	          model_objects_live() == 0,
	      "every external object finalized", why);
	printf("%s\n", why);
	return failures;
}
