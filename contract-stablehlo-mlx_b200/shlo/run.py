"""StablehloMlx/Kernels/Run.lean restated: dispatch the exact kernels.

Each kernel is created once by name (Run.lean:19-25, `"smlx_" ++ name`) and
applied to arrays that stay on the device; the scalar parameters travel as an
8-word uint32 array (Run.lean:51-52). Inputs under 8 elements are padded with
zeros (Run.lean:37-43) -- a Metal binding quirk the CUDA backend does not need,
kept so the call sequence is the reference's.

The Metal source and header strings are not carried: the CUDA backend selects
its kernel by name and ignores them.
"""
from __future__ import annotations

from . import mlx as M

# Binding names per kernel (StablehloMlx/Kernels/Shaders.lean globals).
SPECS = {
    "mul_mat": (["w", "x", "p"], ["y"]),
    "soft_max": (["x", "p"], ["y"]),
    "norm": (["x", "p"], ["y"]),
    "silu": (["x", "p"], ["y"]),
    "gelu_erf": (["x", "erffTable", "p"], ["y"]),
    "erff_map": (["erffTable", "p"], ["y"]),
    "divide": (["a", "b", "p"], ["y"]),
    "sqrt": (["a", "p"], ["y"]),
    "f64_ew": (["a", "b", "p"], ["y"]),
    "f64_of_f32": (["a", "p"], ["y"]),
    "f32_of_f64": (["a", "p"], ["y"]),
}

# This backend's fused forms (no counterpart in the reference): a kernel and
# the built-in adds / multiplies that follow it in one launch, every rounding
# of the unfused sequence kept. The executor uses them when nothing else reads
# the intermediate values.
FUSED = {
    "mul_mat_bias": (["w", "x", "bias", "res", "p"], ["y"]),
    "norm_affine": (["x", "gamma", "beta", "p"], ["y"]),
    "attention": (["q", "k", "v", "p"], ["y"]),
}
EP_BIAS, EP_BIAS_LHS, EP_RES, EP_RES_LHS, EP_GELU = 1, 2, 4, 8, 16

_cache: dict = {}


def kernel(name: str) -> M.Kernel:
    k = _cache.get(name)
    if k is None:
        if name in SPECS:
            ins, outs = SPECS[name]
            k = M.kernel_new("smlx_" + name, ins, outs, "", "")
        elif name in FUSED:
            ins, outs = FUSED[name]
            k = M.kernel_new("shlo_" + name, ins, outs, "", "")
        else:
            raise M.ShloError("no generated kernel %s" % name)
        _cache[name] = k
    return k


def run(name: str, inputs, out_shape, out_dtype: int, threads: int, tg: int) -> M.Arr:
    """Run.lean:34-45."""
    k = kernel(name)
    padded = []
    for a in inputs:
        n = 1
        for d in M.shape(a):
            n *= d
        if n >= 8:
            padded.append(a)
            continue
        pad = M.astype(M.u32_arr([0] * (8 - n)), M.dtype(a))
        padded.append(M.concat([M.reshape(a, [n]), pad], 0))
    outs = M.kernel_apply(k, padded, [out_shape], bytes([out_dtype]), [max(threads, 1), 1, 1], [tg, 1, 1])
    return outs[0]


def params(ws) -> M.Arr:
    """Run.lean:51-52: the parameter words, padded to 8."""
    ws = list(ws) + [0] * (8 - len(ws))
    return M.u32_arr(ws)


_erff_table = None


def erff_table() -> M.Arr:
    """Run.lean:54-60 binds a coefficient table here; the correctly rounded erff
    of this backend needs none, so the binding gets a placeholder of 8 zeros."""
    global _erff_table
    if _erff_table is None:
        _erff_table = M.of_bytes(bytes(32), [8], M.dtF32)
    return _erff_table


def mul_mat(w, x, K, M_, R, N, w_batch_stride, plain=False):
    """Run.lean:62-65: ggml_mul_mat's dot order; w is [Wb, M, K], x is [R, K] with
    R = batch * N; the result is [R, M]."""
    return run("mul_mat", [w, x, params([K, M_, R, w_batch_stride, N, 1 if plain else 0])], [R * M_], M.dtF32,
               R * M_, 64)


def soft_max(x, ncols, rows, scale_bits, float_sum=False):
    return run("soft_max", [x, params([ncols, rows, scale_bits, 1 if float_sum else 0])], [rows * ncols], M.dtF32,
               rows, 64)


def norm(x, ncols, rows, eps_bits, gpu_ops=False):
    return run("norm", [x, params([ncols, rows, eps_bits, 1 if gpu_ops else 0])], [rows * ncols], M.dtF32, rows, 64)


def silu(x, count, gpu_ops=False):
    return run("silu", [x, params([count, 1 if gpu_ops else 0])], [count], M.dtF32, count, 64)


def gelu_erf(x, count, gpu_erf=False):
    return run("gelu_erf", [x, erff_table(), params([count, 1 if gpu_erf else 0])], [count], M.dtF32, count, 64)


def erff_map(base, count):
    return run("erff_map", [erff_table(), params([base, count])], [count], M.dtU32, count, 256)


def divide(a, b, count):
    return run("divide", [a, b, params([count])], [count], M.dtF32, count, 256)


def sqrt(a, count):
    return run("sqrt", [a, params([count])], [count], M.dtF32, count, 256)


F64_ADD, F64_SUB, F64_MUL, F64_DIV, F64_FLOOR, F64_TO_I64 = range(6)


def f64_ew(op, a, b, count):
    return run("f64_ew", [a, b, params([count, op])], [count], M.dtU64, count, 256)


def f64_of_f32(a, count):
    return run("f64_of_f32", [a, params([count])], [count], M.dtU64, count, 256)


def f32_of_f64(a, count):
    return run("f32_of_f64", [a, params([count])], [count], M.dtF32, count, 256)


def mul_mat_bias(w, x, K, M_, R, N, w_batch_stride, bias, res=None, flags=EP_BIAS):
    """mul_mat, then + bias[m] (and + res[r][m] when EP_RES is in flags), each
    add rounded alone in the module's operand order (EP_*_LHS: the added
    value is the add's left operand), then gelu_erf when EP_GELU is in flags."""
    return run("mul_mat_bias", [w, x, bias, res if res is not None else bias,
                                params([K, M_, R, w_batch_stride, N, 0, flags])], [R * M_], M.dtF32, R * M_, 64)


def norm_affine(x, ncols, rows, eps_bits, gamma, beta):
    """norm, then (y * gamma[c]) + beta[c], each rounded alone."""
    return run("norm_affine", [x, gamma, beta, params([ncols, rows, eps_bits, 0])], [rows * ncols], M.dtF32, rows, 64)


def attention(q, k, v, B, S, H, W, scale_bits):
    """q, k, v [B, S, H, W] (any strides): per (batch, head) mul_mat(k, q)
    (the scores, K = W), soft_max(scale), mul_mat(v^T, p) (K = S), the result
    [B, S, H, W] -- the transposed layout of the merged heads."""
    return run("attention", [q, k, v, params([B, S, H, W, scale_bits])], [B * S * H * W], M.dtF32, B * S * H, 64)
