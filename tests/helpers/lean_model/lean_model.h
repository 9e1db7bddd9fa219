/* Helpers of the Lean runtime model (lean_model.c) that Lean itself spells
   differently: closures from C functions, byte and Nat arrays, counters. Test
   infrastructure only. */
#pragma once
#include <stddef.h>
#include <stdint.h>

#include <lean/lean.h>

/* A closure `Array Arr -> IO (Array Arr)`: called with (env, args, world), both
   arguments owned by the callee, returning an IO result. */
typedef lean_object *(*model_closure_fn)(void *env, lean_object *args, lean_object *world);
lean_object *model_closure(model_closure_fn fn, void *env);
/* A ByteArray holding a copy of `n` bytes. */
lean_object *model_bytes(const void *data, size_t n);
/* An Array Nat. */
lean_object *model_nats(const int64_t *v, int n);
/* The message of an IO error result (NULL for an ok result). */
const char *model_error_text(b_lean_obj_arg r);
/* IO.Error.toString, which the Lean runtime exports. */
lean_object *lean_io_error_to_string(lean_object *err);

long model_objects_live(void);
long model_externals_made(void);
long model_externals_finalized(void);
