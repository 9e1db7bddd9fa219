/* A small working model of the Lean 4 runtime objects that
 * contract-stablehlo-mlx_b200/csrc/shlo_cuda_lean.c touches -- test
 * infrastructure only, written here (not Lean's runtime), so the glue can be
 * linked and run where Lean is not installed.
 *
 * It implements the declarations of tests/helpers/lean_stub/lean/lean.h with
 * the semantics the glue relies on: reference counts (lean_inc / lean_dec, an
 * object freed at zero with its children), scalars boxed as tagged pointers,
 * arrays that lean_array_push consumes and returns, byte arrays, strings,
 * external objects whose class finalizer runs when the last reference goes,
 * IO results (ok / error) and user errors, and closures applied with
 * lean_apply_2 (which consumes the closure and its arguments). Counters let a
 * test check that every external object was finalized.
 */
#define _POSIX_C_SOURCE 200809L
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <lean/lean.h>

#include "lean_model.h"

enum kind { K_EXTERNAL = 1, K_ARRAY, K_SARRAY, K_STRING, K_RESULT, K_USER_ERROR, K_CLOSURE };

struct lean_external_class {
	lean_external_finalize_proc finalize;
	lean_external_foreach_proc foreach;
};

struct lean_object {
	int rc;
	int kind;
	int tag;  /* K_RESULT: 0 ok, 1 error */
	/* K_EXTERNAL */
	lean_external_class *cls;
	void *data;
	/* K_ARRAY */
	lean_object **items;
	size_t size, cap;
	/* K_SARRAY */
	uint8_t *bytes;
	/* K_STRING */
	char *str;
	/* K_RESULT, K_USER_ERROR: one field */
	lean_object *field;
	/* K_CLOSURE */
	model_closure_fn fn;
	void *env;
};

static long g_objects_live, g_externals_made, g_externals_finalized;

static int is_scalar(const lean_object *o) { return ((uintptr_t)o & 1) != 0; }

static lean_object *new_obj(int kind) {
	lean_object *o = (lean_object *)calloc(1, sizeof(lean_object));
	if (!o) {
		fprintf(stderr, "lean model: out of memory\n");
		abort();
	}
	o->rc = 1;
	o->kind = kind;
	g_objects_live++;
	return o;
}

void lean_inc(lean_object *o) {
	if (o && !is_scalar(o)) o->rc++;
}

void lean_dec(lean_object *o) {
	if (!o || is_scalar(o)) return;
	if (--o->rc > 0) return;
	switch (o->kind) {
		case K_EXTERNAL:
			if (o->cls && o->cls->finalize) o->cls->finalize(o->data);
			g_externals_finalized++;
			break;
		case K_ARRAY:
			for (size_t i = 0; i < o->size; i++) lean_dec(o->items[i]);
			free(o->items);
			break;
		case K_SARRAY: free(o->bytes); break;
		case K_STRING: free(o->str); break;
		case K_RESULT:
		case K_USER_ERROR: lean_dec(o->field); break;
		case K_CLOSURE: break;
	}
	g_objects_live--;
	free(o);
}

lean_external_class *lean_register_external_class(lean_external_finalize_proc fin, lean_external_foreach_proc fe) {
	lean_external_class *c = (lean_external_class *)calloc(1, sizeof(lean_external_class));
	c->finalize = fin;
	c->foreach = fe;
	return c;
}

lean_object *lean_alloc_external(lean_external_class *cls, void *data) {
	lean_object *o = new_obj(K_EXTERNAL);
	o->cls = cls;
	o->data = data;
	g_externals_made++;
	return o;
}

void *lean_get_external_data(b_lean_obj_arg o) { return o->data; }

size_t lean_array_size(b_lean_obj_arg o) { return o->size; }

lean_object *lean_array_get_core(b_lean_obj_arg o, size_t i) { return o->items[i]; }

lean_object *lean_alloc_array(size_t size, size_t cap) {
	lean_object *o = new_obj(K_ARRAY);
	o->cap = cap > size ? cap : size;
	o->items = (lean_object **)calloc(o->cap ? o->cap : 1, sizeof(lean_object *));
	o->size = size;
	return o;
}

lean_object *lean_array_push(lean_obj_arg a, lean_obj_arg v) {
	if (a->size == a->cap) {
		a->cap = a->cap ? 2 * a->cap : 4;
		a->items = (lean_object **)realloc(a->items, a->cap * sizeof(lean_object *));
	}
	a->items[a->size++] = v;
	return a;
}

size_t lean_unbox(b_lean_obj_arg o) { return (size_t)((uintptr_t)o >> 1); }

lean_object *lean_box(size_t n) { return (lean_object *)(uintptr_t)((n << 1) | 1); }

lean_object *lean_uint64_to_nat(uint64_t n) {
	if (n >> 62) {
		fprintf(stderr, "lean model: a natural number above 2^62 is not modelled\n");
		abort();
	}
	return lean_box((size_t)n);
}

uint8_t *lean_sarray_cptr(lean_object *o) { return o->bytes; }

size_t lean_sarray_size(b_lean_obj_arg o) { return o->size; }

lean_object *lean_alloc_sarray(unsigned elem, size_t size, size_t cap) {
	lean_object *o = new_obj(K_SARRAY);
	size_t n = (size_t)elem * (cap > size ? cap : size);
	o->bytes = (uint8_t *)calloc(n ? n : 1, 1);
	o->size = size;
	o->cap = cap;
	return o;
}

const char *lean_string_cstr(b_lean_obj_arg o) { return o->str; }

lean_object *lean_mk_string(const char *s) {
	lean_object *o = new_obj(K_STRING);
	o->str = strdup(s ? s : "");
	return o;
}

lean_object *lean_mk_io_user_error(lean_obj_arg msg) {
	lean_object *o = new_obj(K_USER_ERROR);
	o->field = msg;
	return o;
}

static lean_object *result(int tag, lean_object *v) {
	lean_object *o = new_obj(K_RESULT);
	o->tag = tag;
	o->field = v;
	return o;
}

lean_obj_res lean_io_result_mk_error(lean_obj_arg e) { return result(1, e); }
lean_obj_res lean_io_result_mk_ok(lean_obj_arg v) { return result(0, v); }
int lean_io_result_is_error(b_lean_obj_arg r) { return r->kind == K_RESULT && r->tag == 1; }
lean_object *lean_io_result_get_error(b_lean_obj_arg r) { return r->field; }
lean_object *lean_io_result_get_value(b_lean_obj_arg r) { return r->field; }
lean_object *lean_io_mk_world(void) { return lean_box(0); }

lean_object *lean_io_error_to_string(lean_object *err) {
	lean_object *s;
	if (err->kind == K_USER_ERROR && !is_scalar(err->field) && err->field->kind == K_STRING) {
		s = err->field;
		lean_inc(s);
	} else {
		s = lean_mk_string("(an IO error the model does not print)");
	}
	lean_dec(err);
	return s;
}

lean_object *lean_apply_2(lean_object *f, lean_object *a, lean_object *b) {
	lean_object *r = f->fn(f->env, a, b);
	lean_dec(f);
	return r;
}

/* ---- the model's own helpers ---- */

lean_object *model_closure(model_closure_fn fn, void *env) {
	lean_object *o = new_obj(K_CLOSURE);
	o->fn = fn;
	o->env = env;
	return o;
}

lean_object *model_bytes(const void *data, size_t n) {
	lean_object *o = lean_alloc_sarray(1, n, n);
	if (n) memcpy(o->bytes, data, n);
	return o;
}

lean_object *model_nats(const int64_t *v, int n) {
	lean_object *a = lean_alloc_array(0, (size_t)n);
	for (int i = 0; i < n; i++) a = lean_array_push(a, lean_box((size_t)v[i]));
	return a;
}

const char *model_error_text(b_lean_obj_arg r) {
	if (!lean_io_result_is_error(r)) return NULL;
	lean_object *e = r->field;
	if (e->kind == K_USER_ERROR && !is_scalar(e->field) && e->field->kind == K_STRING) return e->field->str;
	return "(an IO error the model does not print)";
}

long model_objects_live(void) { return g_objects_live; }
long model_externals_made(void) { return g_externals_made; }
long model_externals_finalized(void) { return g_externals_finalized; }
