"""The Lean glue (csrc/shlo_cuda_lean.c) defines every symbol the reference's
Lean declarations bind (StablehloMlx/Mlx.lean:16-73) and type-checks against
the lean.h API it uses. Lean itself is not installed here, so this is a
compile-only check against a declaration stub."""
import os
import re
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GLUE = os.path.join(ROOT, "contract-stablehlo-mlx_b200", "csrc", "shlo_cuda_lean.c")

# The @[extern] names of StablehloMlx/Mlx.lean.
SMLX = ["smlx_empty", "smlx_of_bytes", "smlx_to_bytes", "smlx_shape", "smlx_dtype", "smlx_unary", "smlx_binary",
        "smlx_where", "smlx_reshape", "smlx_transpose", "smlx_broadcast", "smlx_slice", "smlx_concat", "smlx_astype",
        "smlx_view", "smlx_take", "smlx_max_axis", "smlx_contiguous", "smlx_eval", "smlx_kernel_new",
        "smlx_kernel_apply", "smlx_compile", "smlx_apply", "smlx_libm_erff_range", "smlx_count_nonzero"]


def test_glue_defines_every_extern():
    text = open(GLUE).read()
    defined = set(re.findall(r"LEAN_EXPORT lean_obj_res (smlx_\w+)\(", text))
    defined |= set(re.findall(r"SHAPE_OP\((smlx_\w+),", text))
    assert sorted(defined) == sorted(SMLX)


def test_glue_type_checks():
    stub = os.path.join(ROOT, "tests", "helpers", "lean_stub")
    r = subprocess.run(["/usr/bin/gcc", "-fsyntax-only", "-Wall", "-Werror", "-std=c11", "-I", stub, GLUE],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
