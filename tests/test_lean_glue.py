"""The Lean glue (csrc/shlo_cuda_lean.c) defines every symbol the reference's
Lean declarations bind (StablehloMlx/Mlx.lean:16-73), type-checks against the
lean.h API it uses, and runs: Lean itself is not installed here, so the glue is
linked against a small model of the Lean runtime's objects
(tests/helpers/lean_model/) and driven the way the Lean executor drives it."""
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


# ---- the glue linked and run: tests/helpers/lean_model/ models the Lean
# runtime objects the glue touches, and lean_glue_run drives the glue as the
# Lean executor would (Run.lean's mulMat, Mlx.lean's compile/apply).

import hashlib  # noqa: E402

import numpy as np  # noqa: E402
import pytest  # noqa: E402

MODEL = os.path.join(ROOT, "tests", "helpers", "lean_model")
LIB_DIR = os.path.join(ROOT, "contract-stablehlo-mlx_b200", "lib")


def build_runner(tmp):
    exe = os.path.join(str(tmp), "lean_glue_run")
    cmd = ["/usr/bin/gcc", "-std=c11", "-Wall", "-Werror", "-O1", "-I", os.path.join(ROOT, "tests", "helpers", "lean_stub"),
           "-I", MODEL, os.path.join(MODEL, "lean_model.c"), os.path.join(MODEL, "lean_glue_run.c"), GLUE,
           "-L", LIB_DIR, "-lshlo_cuda", "-Wl,-rpath," + LIB_DIR, "-o", exe]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_glue_runs_without_gpu(tmp_path):
    """Error paths and finalizers: an unknown kernel is refused as not carried,
    a failing traced function's message comes back through apply, a glue-side
    check (nine outputs, a two-entry grid) reports its own message, and every
    external object is finalized once its references are gone."""
    exe = build_runner(tmp_path)
    r = subprocess.run([exe, "cpu"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "FAIL" not in r.stdout


@pytest.mark.gpu
def test_glue_runs_the_kernel_path(tmp_path, pins):
    """ofBytes -> kernelNew "smlx_mul_mat" -> kernelApply -> toBytes through the
    glue, eager and inside a compiled function (recorded, then replayed), on the
    ggml case mul_mat_small (its pinned SHA-256) and on a packed-path shape
    (the oracle)."""
    from oracle import ggml_cases as G
    from oracle import oracle as O

    exe = build_runner(tmp_path)
    c = G.BY_NAME["mul_mat_small"]
    w, x = c.inputs()
    K, Mm, R = c.extra["K"], c.extra["M"], c.extra["R"] * c.extra["B"]
    rng = np.random.default_rng(5)
    cases = [("small", w.reshape(Mm, K), x.reshape(R, K), K, Mm, R, pins["pinned"]["mul_mat_small/out.f32"]),
             ("packed", rng.standard_normal((256, 512)).astype(np.float32),
              rng.standard_normal((96, 512)).astype(np.float32), 512, 256, 96, None)]
    for name, wa, xa, k, m, r_, pin in cases:
        d = tmp_path / name
        d.mkdir()
        wa.astype(np.float32).tofile(str(d / "w.f32"))
        xa.astype(np.float32).tofile(str(d / "x.f32"))
        env = dict(os.environ, SHLO_GGML_FLAVOR="pinned")
        r = subprocess.run([exe, "gpu", str(d), str(k), str(m), str(r_)], capture_output=True, text=True, timeout=300,
                           env=env)
        assert r.returncode == 0, r.stdout + r.stderr
        outs = [(d / f).read_bytes() for f in ("out_eager.f32", "out_compiled.f32", "out_replay.f32")]
        assert outs[0] == outs[1] == outs[2]
        if pin is not None:
            assert hashlib.sha256(outs[0]).hexdigest() == pin
        else:
            want = O.mul_mat(wa, xa, k, m, r_, r_, 0, O.PINNED)
            assert outs[0] == want.tobytes()
