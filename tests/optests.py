"""Tests/OpTests.lean restated for the replay harness: the module text of each
ggml case (OpTests.lean:32-106) and the case list with its planted fault
(OpTests.lean:118-139). Test infrastructure only."""
from __future__ import annotations

import struct
from dataclasses import dataclass, field

from shlo import lower as L


def ty_of(ne) -> L.Ty:
    """ggml `ne` (fastest first) as a rank-3 MLIR type (slowest first)."""
    return L.Ty((ne[2], ne[1], ne[0]), "f32")


def hex32(b: int) -> str:
    return "0x%08X" % (b & 0xFFFFFFFF)


def fn_header(args, outs) -> str:
    return ("module {\n  func.func public @main(" + ", ".join("%%a%d: %s" % (i, t.str()) for i, t in enumerate(args))
            + ") -> (" + ", ".join(t.str() for t in outs) + ") {\n")


def fn_footer(r: str, t: L.Ty) -> str:
    return "    func.return %s : %s\n  }\n}\n" % (r, t.str())


def unary_call(target: str, attrs: str, t: L.Ty) -> str:
    return (fn_header([t], [t]) + '    %%0 = "stablehlo.custom_call"(%%a0) {call_target_name = "%s", backend_config = "%s"} : (%s) -> %s\n'
            % (target, attrs, t.str(), t.str()) + fn_footer("%0", t))


def scale_bits() -> int:
    """1.0f / sqrtf(128.0f) in binary32 (ggml_ref.c:193)."""
    import numpy as np
    v = np.float32(1.0) / np.sqrt(np.float32(128.0))
    return struct.unpack("<I", struct.pack("<f", float(v)))[0]


def module_for(op: str, ins, out) -> str:
    to = ty_of(out)
    if op == "mul_mat":
        w, x = ins
        tw, tx = ty_of(w), ty_of(x)
        tr = L.Ty((x[2], x[1], w[2], w[1]), "f32")
        return (fn_header([tw, tx], [to]) +
                '    %%0 = "stablehlo.dot_general"(%%a1, %%a0) {dot_dimension_numbers = #stablehlo.dot<lhs_contracting_dimensions = [2], rhs_contracting_dimensions = [2]>} : (%s, %s) -> %s\n'
                % (tx.str(), tw.str(), tr.str()) +
                '    %%1 = "stablehlo.reshape"(%%0) : (%s) -> %s\n' % (tr.str(), to.str()) + fn_footer("%1", to))
    if op in ("add", "mul"):
        n = "stablehlo.add" if op == "add" else "stablehlo.multiply"
        return (fn_header([to, to], [to]) + '    %%0 = "%s"(%%a0, %%a1) : (%s, %s) -> %s\n' % (n, to.str(), to.str(), to.str())
                + fn_footer("%0", to))
    if op == "repeat":
        ti = ty_of(ins[0])
        return (fn_header([ti], [to]) +
                '    %%0 = "stablehlo.broadcast_in_dim"(%%a0) {broadcast_dimensions = array<i64: 0, 1, 2>} : (%s) -> %s\n'
                % (ti.str(), to.str()) + fn_footer("%0", to))
    if op == "scale":
        st = L.Ty((), "f32")
        return (fn_header([to], [to]) +
                '    %%0 = "stablehlo.constant"() {value = dense<%s> : tensor<f32>} : () -> tensor<f32>\n' % hex32(scale_bits()) +
                '    %%1 = "stablehlo.broadcast_in_dim"(%%0) {broadcast_dimensions = array<i64>} : (%s) -> %s\n' % (st.str(), to.str()) +
                '    %%2 = "stablehlo.multiply"(%%a0, %%1) : (%s, %s) -> %s\n' % (to.str(), to.str(), to.str()) + fn_footer("%2", to))
    if op == "norm":
        return unary_call("ggml.norm", "eps = 0x3727C5AC : f32", to)
    if op == "soft_max":
        return unary_call("ggml.soft_max", "scale = 0x3F800000 : f32", to)
    if op == "gelu_erf":
        return unary_call("ggml.gelu_erf", "", to)
    if op == "silu":
        return unary_call("ggml.silu", "", to)
    if op.startswith("concat"):
        d = 2 - int(op[6:])
        ta, tb = ty_of(ins[0]), ty_of(ins[1])
        return (fn_header([ta, tb], [to]) +
                '    %%0 = "stablehlo.concatenate"(%%a0, %%a1) {dimension = %d : i64} : (%s, %s) -> %s\n' % (d, ta.str(), tb.str(), to.str())
                + fn_footer("%0", to))
    if op == "transpose":
        ti = ty_of(ins[0])
        return (fn_header([ti], [to]) +
                '    %%0 = "stablehlo.transpose"(%%a0) {permutation = array<i64: 0, 2, 1>} : (%s) -> %s\n' % (ti.str(), to.str())
                + fn_footer("%0", to))
    raise ValueError("no module builder for " + op)


def view_module(inp, out, off: int) -> str:
    ti, to = ty_of(inp), ty_of(out)
    return (fn_header([ti], [to]) +
            '    %%0 = "stablehlo.slice"(%%a0) {start_indices = array<i64: 0, 0, %d>, limit_indices = array<i64: 1, %d, %d>, strides = array<i64: 1, 1, 1>} : (%s) -> %s\n'
            % (off, out[1], off + out[0], ti.str(), to.str()) + fn_footer("%0", to))


@dataclass
class OpCase:
    name: str
    op: str
    fault: L.Faults
    fault_name: str
    view_offset: int = 0
    expect_refusal: bool = False


def cases():
    def mm(n):
        return OpCase(n, "mul_mat", L.Faults(dotBuiltin=True), "built-in matmul")

    def mm_plain(n):
        return OpCase(n, "mul_mat", L.Faults(dotPlain=True), "sequential sum without FMA")

    out = [mm_plain("mul_mat_small"), mm_plain("mul_mat_k2"), mm("mul_mat_qkv"), mm("mul_mat_ffn2"), mm("mul_mat_text"),
           mm_plain("mul_mat_heading"), mm("mul_mat_root_in"), mm("mul_mat_body_in"), mm("mul_mat_scores"),
           mm("mul_mat_value")]
    out += [OpCase(n, "add", L.Faults(binaryHalf=True), "float16 arithmetic") for n in ("add_small", "add_kimodo")]
    out += [OpCase(n, "mul", L.Faults(binaryHalf=True), "float16 arithmetic") for n in ("mul_small", "mul_kimodo")]
    out += [OpCase(n, "scale", L.Faults(binaryHalf=True), "float16 arithmetic") for n in ("scale_small", "scale_kimodo")]
    out += [OpCase(n, "repeat", L.Faults(broadcastFirst=True), "broadcast of the first element")
            for n in ("repeat_small", "repeat_kimodo")]
    out += [OpCase(n, "norm", L.Faults(normGpuOps=True), "binary32 sums and GPU / and sqrt")
            for n in ("norm_small", "norm_kimodo")]
    out += [OpCase(n, "soft_max", L.Faults(softMaxFloatSum=True), "binary32 denominator")
            for n in ("soft_max_small", "soft_max_kimodo")]
    out += [OpCase("soft_max_tail", "soft_max", L.Faults(), "", expect_refusal=True)]
    out += [OpCase(n, "gelu_erf", L.Faults(geluTanh=True), "tanh-form GELU") for n in ("gelu_erf_small", "gelu_erf_kimodo")]
    out += [OpCase(n, "silu", L.Faults(siluGpuOps=True), "GPU exp and /") for n in ("silu_small", "silu_kimodo")]
    out += [OpCase("silu_tail", "silu", L.Faults(), "", expect_refusal=True)]
    out += [OpCase(n, o, L.Faults(concatSwap=True), "operands swapped")
            for n, o in (("concat0_small", "concat0"), ("concat1_small", "concat1"), ("concat2_small", "concat2"),
                         ("concat0_kimodo", "concat0"), ("concat1_kimodo", "concat1"), ("concat2_kimodo", "concat2"))]
    out += [OpCase(n, "transpose", L.Faults(transposeIdentity=True), "no permutation")
            for n in ("transpose_small", "transpose_kimodo")]
    out += [OpCase("view_small", "view", L.Faults(sliceShift=True), "offset one late", view_offset=8),
            OpCase("view_kimodo", "view", L.Faults(sliceShift=True), "offset one late", view_offset=1024 + 3 * 128)]
    return out
