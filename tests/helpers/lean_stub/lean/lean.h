/* A declaration-only stand-in for the subset of Lean 4's lean.h that
   contract-stablehlo-mlx_b200/csrc/shlo_cuda_lean.c uses, so the tests can
   compile the glue where Lean is not installed. tests/helpers/lean_model/
   implements these declarations (a small model of the Lean runtime's objects)
   so that the glue also links and runs. */
#pragma once
#include <stddef.h>
#include <stdint.h>
typedef struct lean_object lean_object;
typedef lean_object *lean_obj_arg;
typedef lean_object *b_lean_obj_arg;
typedef lean_object *lean_obj_res;
typedef struct lean_external_class lean_external_class;
typedef void (*lean_external_finalize_proc)(void *);
typedef void (*lean_external_foreach_proc)(void *, b_lean_obj_arg);
#define LEAN_EXPORT __attribute__((visibility("default")))
lean_external_class *lean_register_external_class(lean_external_finalize_proc, lean_external_foreach_proc);
lean_object *lean_alloc_external(lean_external_class *, void *);
void *lean_get_external_data(b_lean_obj_arg);
size_t lean_array_size(b_lean_obj_arg);
lean_object *lean_array_get_core(b_lean_obj_arg, size_t);
lean_object *lean_alloc_array(size_t, size_t);
lean_object *lean_array_push(lean_obj_arg, lean_obj_arg);
size_t lean_unbox(b_lean_obj_arg);
lean_object *lean_box(size_t);
lean_object *lean_uint64_to_nat(uint64_t);
uint8_t *lean_sarray_cptr(lean_object *);
size_t lean_sarray_size(b_lean_obj_arg);
lean_object *lean_alloc_sarray(unsigned, size_t, size_t);
const char *lean_string_cstr(b_lean_obj_arg);
lean_object *lean_mk_string(const char *);
lean_object *lean_mk_io_user_error(lean_obj_arg);
lean_obj_res lean_io_result_mk_error(lean_obj_arg);
lean_obj_res lean_io_result_mk_ok(lean_obj_arg);
int lean_io_result_is_error(b_lean_obj_arg);
lean_object *lean_io_result_get_error(b_lean_obj_arg);
lean_object *lean_io_result_get_value(b_lean_obj_arg);
lean_object *lean_io_mk_world(void);
lean_object *lean_apply_2(lean_object *, lean_object *, lean_object *);
void lean_inc(lean_object *);
void lean_dec(lean_object *);
