"""StablehloMlx/Lower.lean restated: each StableHLO op as calls of the boundary.

`run_op` follows Lower.lean:334-473 op by op -- the same sequence of
Mlx/Run calls, the same refusals ("not carried"), and the same planted wrong
lowerings (`Faults`, Lower.lean:53-69), so the parity tests drive the CUDA
backend exactly as the Lean executor would. Values are `mlx.Arr`; types are
`Ty(dims, el)` with MLIR element names ("f32", "i64", "ui32", "f64", ...).
"""
from __future__ import annotations

import re
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

from . import mlx as M
from . import run as Run


@dataclass
class Ty:
    dims: tuple
    el: str

    @property
    def count(self) -> int:
        n = 1
        for d in self.dims:
            n *= d
        return n

    def str(self) -> str:
        return "tensor<" + "".join("%dx" % d for d in self.dims) + self.el + ">"


@dataclass
class Faults:
    """Planted wrong lowerings, all off in normal use (Lower.lean:53-69)."""
    dotBuiltin: bool = False
    dotPlain: bool = False
    softMaxFloatSum: bool = False
    normGpuOps: bool = False
    siluGpuOps: bool = False
    geluTanh: bool = False
    divideBuiltin: bool = False
    sqrtBuiltin: bool = False
    binaryHalf: bool = False
    broadcastFirst: bool = False
    concatSwap: bool = False
    transposeIdentity: bool = False
    sliceShift: bool = False
    f64AsF32: bool = False
    whileShort: bool = False


class NotCarried(M.ShloError):
    pass


def err(msg: str):
    raise NotCarried(msg) if "not carried" in msg else M.ShloError(msg)


# ---- attribute text (Lower.lean:80-153) ----

def ints(s: str) -> List[int]:
    """The integers in `array<i64: 1, 2>`, `[1, 2]`, or `dense<[1, 2]> : ...`."""
    if s.startswith("array<"):
        parts = s.split(":")
        body = ":".join(parts[1:]) if len(parts) > 1 else ""
    else:
        body = s
    return [int(t) for t in re.findall(r"\d+", body)]


def field_(s: str, key: str) -> str:
    parts = s.split(key + " = ")
    if len(parts) < 2:
        return ""
    return parts[1].split("]")[0] + "]"


def el_dtype(el: str) -> int:
    table = {"f32": M.dtF32, "i32": M.dtI32, "si32": M.dtI32, "ui32": M.dtU32, "i64": M.dtI64, "si64": M.dtI64,
             "ui64": M.dtU64, "i1": M.dtBool, "ui8": M.dtU8, "f64": M.dtU64}
    if el not in table:
        err("element type %s is not carried" % el)
    return table[el]


def el_bytes(el: str) -> int:
    if el in ("f64", "i64", "ui64", "si64"):
        return 8
    if el in ("i1", "ui8"):
        return 1
    return 4


def literal_bits(el: str, lit: str) -> int:
    t = lit.strip()
    if t == "true":
        return 1
    if t == "false":
        return 0
    if t.lower().startswith("0x"):
        return int(t[2:], 16)
    if el.startswith("f"):
        err("decimal float literal %s for %s: write it as a hex bit pattern so it is exact" % (t, el))
    v = int(t)
    w = 8 * el_bytes(el)
    return (v + (1 << w)) % (1 << w) if v < 0 else v


def bytes_of(el: str, bits: Sequence[int]) -> bytes:
    w = el_bytes(el)
    return b"".join(int(x).to_bytes(w, "little") for x in bits)


def f32_attr(attrs: str, key: str) -> int:
    parts = attrs.split(key + " = ")
    if len(parts) < 2:
        err("composite attribute %s missing" % key)
    return literal_bits("f32", parts[1].split(" ")[0])


def constant(value: str, t: Ty) -> M.Arr:
    """Lower.lean:134-147."""
    inner = value.split("dense<")[1].split(">")[0] if "dense<" in value else ""
    inner = inner.replace("[", "").replace("]", "")
    lits = [x for x in inner.split(",") if x.strip()]
    bits = [literal_bits(t.el, x) for x in lits]
    dt = el_dtype(t.el)
    if len(bits) == 1 and t.count != 1:
        s = M.of_bytes(bytes_of(t.el, bits), [], dt)
        return M.broadcast(s, list(t.dims))
    if len(bits) != t.count:
        err("constant has %d values for %s" % (len(bits), t.str()))
    return M.of_bytes(bytes_of(t.el, bits), list(t.dims), dt)


# ---- dot_general (Lower.lean:157-182) ----

def dot_general(f: Faults, dn: str, a: M.Arr, b: M.Arr, ta: Ty, tb: Ty, out: Ty) -> M.Arr:
    lb = ints(field_(dn, "lhs_batching_dimensions"))
    rb = ints(field_(dn, "rhs_batching_dimensions"))
    lc = ints(field_(dn, "lhs_contracting_dimensions"))
    rc = ints(field_(dn, "rhs_contracting_dimensions"))
    if len(lc) != 1 or len(rc) != 1:
        err("dot_general: one contracting dimension is carried")
    lf = [d for d in range(len(ta.dims)) if d not in lb and d not in lc]
    rf = [d for d in range(len(tb.dims)) if d not in rb and d not in rc]

    def prod(t, ds):
        n = 1
        for d in ds:
            n *= t.dims[d]
        return n

    B, N, Mm, K = prod(ta, lb), prod(ta, lf), prod(tb, rf), ta.dims[lc[0]]
    a2 = M.reshape(M.transpose(a, lb + lf + lc), [B * N, K])
    b2 = M.reshape(M.transpose(b, rb + rf + rc), [B * Mm, K])
    if f.dotBuiltin:
        a3 = M.reshape(a2, [B, N, K])
        b3 = M.transpose(M.reshape(b2, [B, Mm, K]), [0, 2, 1])
        return M.reshape(M.binary(M.opMatmul, a3, b3), list(out.dims))
    y = Run.mul_mat(b2, a2, K, Mm, B * N, N, Mm * K if B > 1 else 0, f.dotPlain)
    return M.reshape(y, list(out.dims))


# ---- the table (Lower.lean:186-219) ----

UNARY = {"stablehlo.negate": M.opNeg, "stablehlo.abs": M.opAbs, "stablehlo.floor": M.opFloor,
         "stablehlo.not": M.opInvert, "stablehlo.exponential": M.opExp, "stablehlo.tanh": M.opTanh,
         "stablehlo.logistic": M.opSigmoid}
BINARY = {"stablehlo.add": M.opAdd, "stablehlo.subtract": M.opSub, "stablehlo.multiply": M.opMul,
          "stablehlo.maximum": M.opMax, "stablehlo.minimum": M.opMin, "stablehlo.and": M.opAnd,
          "stablehlo.or": M.opOr, "stablehlo.xor": M.opXor, "stablehlo.shift_left": M.opShl,
          "stablehlo.shift_right_logical": M.opShr, "stablehlo.remainder": M.opRem}


def direction(attr: str) -> str:
    return attr.split("comparison_direction ")[-1].replace(">", "").strip()


def compare_code(d: str) -> int:
    for k, v in (("EQ", M.opEq), ("NE", M.opNe), ("LT", M.opLt), ("LE", M.opLe), ("GT", M.opGt), ("GE", M.opGe)):
        if d.endswith(k):
            return v
    err("comparison %s" % d)


# ---- binary64 as uint64 bit patterns (Lower.lean:255-298) ----

ABS64, INF64, SIGN64, QUIET64 = 0x7FFFFFFFFFFFFFFF, 0x7FF0000000000000, 0x8000000000000000, 0x0008000000000000


def f64_ew(op: int, a: M.Arr, b: M.Arr, t: Ty) -> M.Arr:
    return M.reshape(Run.f64_ew(op, M.reshape(a, [t.count]), M.reshape(b, [t.count]), t.count), list(t.dims))


def f64_nan(x):
    return M.binary(M.opGt, M.binary(M.opAnd, x, M.u64_scalar(ABS64)), M.u64_scalar(INF64))


def f64_zero(x):
    return M.binary(M.opEq, M.binary(M.opAnd, x, M.u64_scalar(ABS64)), M.u64_scalar(0))


def f64_key(x):
    neg = M.binary(M.opMul, M.binary(M.opShr, x, M.u64_scalar(63)), M.u64_scalar(0xFFFFFFFFFFFFFFFF))
    return M.binary(M.opXor, x, M.binary(M.opOr, neg, M.u64_scalar(SIGN64)))


def f64_compare(d: str, a, b):
    ordered = M.binary(M.opLAnd, M.unary(M.opNot, f64_nan(a)), M.unary(M.opNot, f64_nan(b)))
    zeros = M.binary(M.opLAnd, f64_zero(a), f64_zero(b))
    ka, kb = f64_key(a), f64_key(b)
    eq = M.binary(M.opLAnd, ordered, M.binary(M.opLOr, M.binary(M.opEq, a, b), zeros))
    lt = M.binary(M.opLAnd, ordered, M.binary(M.opLAnd, M.unary(M.opNot, zeros), M.binary(M.opLt, ka, kb)))
    gt = M.binary(M.opLAnd, ordered, M.binary(M.opLAnd, M.unary(M.opNot, zeros), M.binary(M.opGt, ka, kb)))
    if d.endswith("EQ"):
        return eq
    if d.endswith("NE"):
        return M.unary(M.opNot, eq)
    if d.endswith("LT"):
        return lt
    if d.endswith("LE"):
        return M.binary(M.opLOr, lt, eq)
    if d.endswith("GT"):
        return gt
    if d.endswith("GE"):
        return M.binary(M.opLOr, gt, eq)
    err("comparison %s" % d)


def f64_max_min(is_max: bool, a, b):
    def q(x):
        return M.binary(M.opOr, x, M.u64_scalar(QUIET64))
    pick = M.binary(M.opGe if is_max else M.opLe, f64_key(a), f64_key(b))
    r = M.where_(pick, a, b)
    return M.where_(f64_nan(a), q(a), M.where_(f64_nan(b), q(b), r))


def rows_cols(t: Ty):
    c = t.dims[-1] if t.dims else 1
    return (t.count // max(c, 1), c)


def convert_op(a, src: Ty, out: Ty):
    """Lower.lean:306-315."""
    s, e = src.el, out.el
    if s == "f32" and e == "f64":
        return M.reshape(Run.f64_of_f32(M.reshape(a, [out.count]), out.count), list(out.dims))
    if s == "f64" and e == "f32":
        return M.reshape(Run.f32_of_f64(M.reshape(a, [out.count]), out.count), list(out.dims))
    if s == "f64" and e == "f64":
        return a
    if s == "f64":
        if e in ("i64", "si64"):
            return f64_ew(Run.F64_TO_I64, a, a, out)
        err("convert f64 to %s is not carried" % e)
    if e == "f64":
        err("convert %s to f64 is not carried" % s)
    return M.astype(a, el_dtype(e))


INT_ELS = ("i1", "i8", "ui8", "i32", "si32", "ui32", "i64", "si64", "ui64")


def const_eval(known: Dict[str, int], o) -> Optional[int]:
    """Lower.lean:225-251: the value of a scalar integer that is a constant, or
    arithmetic on such scalars -- what `while` conditions and `dynamic_slice`
    starts are made of (None when it depends on data)."""
    if not o.out_tys or o.out_tys[0].dims != () or o.out_tys[0].el not in INT_ELS:
        return None

    def k(i):
        return known.get(o.operands[i]) if i < len(o.operands) else None
    n = o.name
    if n == "stablehlo.constant":
        v = o.attr("value")
        if v is None:
            return None
        t = (v.split("dense<")[1] if "dense<" in v else "").split(">")[0].strip()
        if t == "true":
            return 1
        if t == "false":
            return 0
        try:
            return int(t)
        except ValueError:
            return None
    if n in ("stablehlo.add", "stablehlo.subtract", "stablehlo.multiply"):
        a, b = k(0), k(1)
        if a is None or b is None:
            return None
        return a + b if n.endswith("add") else a - b if n.endswith("subtract") else a * b
    if n == "stablehlo.convert":
        return k(0)
    if n == "stablehlo.compare":
        a, b = k(0), k(1)
        if a is None or b is None:
            return None
        d = direction(o.attr("comparison_direction") or "")
        r = {"EQ": a == b, "NE": a != b, "LT": a < b, "LE": a <= b, "GT": a > b}.get(d[-2:], a >= b)
        return 1 if r else 0
    return None


def gather1d(o, table: M.Arr, idx: M.Arr) -> M.Arr:
    """Lower.lean:317-331: `stablehlo.gather` of a 1-D table indexed elementwise,
    out[i] = table[clamp(idx[i])] -- the form contract-ggml-stablehlo emits;
    any other form is refused."""
    dn = o.attr("dimension_numbers") or ""
    t, it = o.in_tys[0], o.in_tys[1]
    if not (len(t.dims) == 1 and field_(dn, "collapsed_slice_dims") == "[0]" and field_(dn, "start_index_map") == "[0]"
            and ("index_vector_dim = %d" % len(it.dims)) in dn and ints(o.attr("slice_sizes") or "") == [1]):
        err("gather: only a 1-D table indexed elementwise is carried (%s)" % dn)
    ix = M.astype(idx, M.dtI64)
    lo = M.astype(M.u32_arr([0]), M.dtI64)
    hi = M.astype(M.u32_arr([t.dims[0] - 1]), M.dtI64)
    ix = M.binary(M.opMin, M.binary(M.opMax, ix, M.reshape(lo, [])), M.reshape(hi, []))
    return M.take(table, ix, 0)


@dataclass
class Op:
    """One StableHLO op as the Lean AST holds it (StablehloMlx/Ast.lean)."""
    name: str
    operands: List[str]
    results: List[str]
    attrs: Dict[str, str]
    in_tys: List[Ty]
    out_tys: List[Ty]
    regions: list = field(default_factory=list)

    def attr(self, k: str) -> Optional[str]:
        return self.attrs.get(k)


def run_op(f: Faults, o: Op, args: List[M.Arr], module=None, env=None, known=None) -> List[M.Arr]:
    """Lower.lean:334-473. `env` and `known` are the enclosing values and the
    trace-time integer scalars among them (a region reads the values defined
    around it; `while` and `dynamic_slice` need the scalars)."""
    env = env if env is not None else {}
    known = known if known is not None else {}
    out = o.out_tys[0] if o.out_tys else Ty((), "")
    n = o.name
    el0 = o.in_tys[0].el if o.in_tys else ""
    if el0 == "f64" and f.f64AsF32:
        def narrow(a):
            return convert_op(a, Ty(out.dims, "f64"), Ty(out.dims, "f32"))

        def widen(a):
            return convert_op(a, Ty(out.dims, "f32"), Ty(out.dims, "f64"))
        if n in ("stablehlo.add", "stablehlo.subtract", "stablehlo.multiply"):
            return [widen(M.binary(BINARY[n], narrow(args[0]), narrow(args[1])))]
        if n == "stablehlo.divide":
            return [widen(M.binary(M.opDiv, narrow(args[0]), narrow(args[1])))]
    if el0 == "f64":
        ops = {"stablehlo.add": Run.F64_ADD, "stablehlo.subtract": Run.F64_SUB, "stablehlo.multiply": Run.F64_MUL,
               "stablehlo.divide": Run.F64_DIV}
        if n in ops:
            return [f64_ew(ops[n], args[0], args[1], out)]
        if n == "stablehlo.floor":
            return [f64_ew(Run.F64_FLOOR, args[0], args[0], out)]
        if n == "stablehlo.maximum":
            return [f64_max_min(True, args[0], args[1])]
        if n == "stablehlo.minimum":
            return [f64_max_min(False, args[0], args[1])]
        if n == "stablehlo.abs":
            return [M.binary(M.opAnd, args[0], M.u64_scalar(ABS64))]
        if n == "stablehlo.negate":
            return [M.binary(M.opXor, args[0], M.u64_scalar(SIGN64))]
        if n == "stablehlo.compare":
            return [f64_compare(direction(o.attr("comparison_direction") or ""), args[0], args[1])]
        if n in ("stablehlo.sqrt", "stablehlo.exponential", "stablehlo.tanh", "stablehlo.logistic",
                 "stablehlo.remainder"):
            err("%s on f64 is not carried" % n)
    if el0 == "i1":
        if n == "stablehlo.and":
            return [M.binary(M.opLAnd, args[0], args[1])]
        if n == "stablehlo.or":
            return [M.binary(M.opLOr, args[0], args[1])]
        if n == "stablehlo.xor":
            return [M.binary(M.opNe, args[0], args[1])]
        if n == "stablehlo.not":
            return [M.unary(M.opNot, args[0])]
    if n == "stablehlo.shift_right_logical" and not el0.startswith("ui"):
        err("shift_right_logical on %s (a signed type) is not carried" % el0)
    if n in UNARY:
        return [M.unary(UNARY[n], args[0])]
    if n in BINARY:
        if f.binaryHalf and out.el == "f32":
            def h(a):
                return M.astype(a, M.dtF16)
            return [M.astype(M.binary(BINARY[n], h(args[0]), h(args[1])), M.dtF32)]
        return [M.binary(BINARY[n], args[0], args[1])]
    if n == "stablehlo.constant":
        return [constant(o.attr("value") or err("constant without value"), out)]
    if n == "stablehlo.divide":
        if out.el == "f32" and not f.divideBuiltin:
            return [M.reshape(Run.divide(args[0], args[1], out.count), list(out.dims))]
        return [M.binary(M.opDiv, args[0], args[1])]
    if n == "stablehlo.sqrt":
        if out.el == "f32" and not f.sqrtBuiltin:
            return [M.reshape(Run.sqrt(args[0], out.count), list(out.dims))]
        return [M.unary(M.opSqrt, args[0])]
    if n == "stablehlo.compare":
        return [M.binary(compare_code(direction(o.attr("comparison_direction") or "")), args[0], args[1])]
    if n == "stablehlo.select":
        return [M.where_(args[0], args[1], args[2])]
    if n == "stablehlo.reshape":
        return [M.reshape(args[0], list(out.dims))]
    if n == "stablehlo.transpose":
        perm = ints(o.attr("permutation") or "")
        if f.transposeIdentity:
            return [M.reshape(args[0], list(out.dims))]
        return [M.transpose(args[0], perm)]
    if n == "stablehlo.broadcast_in_dim":
        mp = ints(o.attr("broadcast_dimensions") or "")
        src = o.in_tys[0]
        if f.broadcastFirst:
            first = M.slice_(M.reshape(args[0], [src.count]), [0], [1], [1])
            return [M.broadcast(M.reshape(first, [1] * len(out.dims)), list(out.dims))]
        shp = [1] * len(out.dims)
        for k, d in enumerate(mp):
            shp[d] = src.dims[k]
        return [M.broadcast(M.reshape(args[0], shp), list(out.dims))]
    if n == "stablehlo.slice":
        st = ints(o.attr("start_indices") or "")
        li = ints(o.attr("limit_indices") or "")
        sd = ints(o.attr("strides") or "") or [1] * len(st)
        if f.sliceShift:
            k = len(st) - 1
            st = st[:k] + [st[k] + 1]
            li = li[:k] + [li[k] + 1]
        return [M.slice_(args[0], st, li, sd)]
    if n == "stablehlo.concatenate":
        d = (ints(o.attr("dimension") or "0") or [0])[0]
        return [M.concat(list(reversed(args)) if f.concatSwap else args, d)]
    if n == "stablehlo.convert":
        return [convert_op(args[0], o.in_tys[0], out)]
    if n == "stablehlo.bitcast_convert":
        return [M.view(args[0], el_dtype(out.el))]
    if n == "stablehlo.iota":
        d = (ints(o.attr("iota_dimension") or "0") or [0])[0]
        ln = out.dims[d]
        base = M.astype(M.u32_arr(list(range(ln))), el_dtype(out.el))
        shp = [1] * len(out.dims)
        shp[d] = ln
        return [M.broadcast(M.reshape(base, shp), list(out.dims))]
    if n == "stablehlo.dot_general":
        return [dot_general(f, o.attr("dot_dimension_numbers") or "", args[0], args[1], o.in_tys[0], o.in_tys[1],
                            out)]
    if n == "stablehlo.dynamic_slice":
        # Lower.lean:417-428: the starts must be known at trace time
        src = o.in_tys[0]
        sizes = ints(o.attr("slice_sizes") or "")
        st = []
        for d, nm in enumerate(o.operands[1:]):
            v = known.get(nm)
            if v is None:
                err("dynamic_slice: start %d (%s) depends on data, which is not carried" % (d, nm))
            # StableHLO clamps each start to [0, dim - size]
            st.append(max(0, min(v, src.dims[d] - sizes[d])))
        return [M.slice_(args[0], st, [a + b for a, b in zip(st, sizes)], [1] * len(st))]
    if n == "stablehlo.gather":
        return [gather1d(o, args[0], args[1])]
    if n == "stablehlo.reduce":
        # Lower.lean:430-440: a single-operand maximum; exact and order-free, the
        # init value takes part like any element
        dims = ints(o.attr("dimensions") or "")
        if not o.regions:
            err("reduce without a body")
        body = o.regions[0]
        if not (len(body.ops) == 1 and body.ops[0].name == "stablehlo.maximum" and len(o.operands) == 2):
            err("reduce: only a single-operand maximum is carried")
        if el0 == "f64":
            err("reduce on f64 is not carried")
        r = args[0]
        for d in sorted(dims, reverse=True):
            r = M.max_axis(r, d)
        return [M.binary(M.opMax, r, args[1])]
    if n == "stablehlo.while":
        # Lower.lean:454-470: unrolled while the trace runs; the condition must be known
        if len(o.regions) < 2:
            err("while without its two regions")
        cond, body = o.regions[0], o.regions[1]
        st = list(args)
        st_k = [known.get(nm) for nm in o.operands]
        prev = st
        while True:
            _, ck = run_region(module, f, env, known, cond, st, st_k)
            c = ck[0] if ck else None
            if c is None:
                err("while: the condition depends on data, which is not carried (the loop is unrolled when traced)")
            if c == 0:
                break
            br, bk = run_region(module, f, env, known, body, st, st_k)
            prev, st, st_k = st, br, bk
        return prev if f.whileShort else st
    if n in ("stablehlo.composite", "stablehlo.custom_call"):
        return run_composite(f, o, args, module)
    err("op %s is not in the lowering table" % n)


def run_composite(f: Faults, o: Op, args: List[M.Arr], module=None) -> List[M.Arr]:
    """Lower.lean:475-498: the ggml.* composites run ggml-cpu's routine."""
    name = (o.attr("name") or o.attr("call_target_name") or "").replace('"', "")
    attrs = o.attr("composite_attributes") or o.attr("backend_config") or ""
    out = o.out_tys[0]
    rows, cols = rows_cols(out)
    if name == "ggml.norm":
        y = Run.norm(args[0], cols, rows, f32_attr(attrs, "eps"), f.normGpuOps)
        return [M.reshape(y, list(out.dims))]
    if name == "ggml.soft_max":
        if cols % 4 != 0:
            err("ggml.soft_max: a row of %d has a %d-element tail that ggml-cpu sends through the platform expf, "
                "which is not carried" % (cols, cols % 4))
        y = Run.soft_max(args[0], cols, rows, f32_attr(attrs, "scale"), f.softMaxFloatSum)
        return [M.reshape(y, list(out.dims))]
    if name == "ggml.silu":
        if cols % 4 != 0:
            err("ggml.silu: a row of %d has a %d-element tail that ggml-cpu sends through the platform expf, "
                "which is not carried" % (cols, cols % 4))
        return [M.reshape(Run.silu(args[0], out.count, f.siluGpuOps), list(out.dims))]
    if name == "ggml.gelu_erf":
        return [M.reshape(Run.gelu_erf(args[0], out.count, f.geluTanh), list(out.dims))]
    if module is not None:
        dec = (o.attr("decomposition") or "").replace("@", "")
        fn = module.funcs.get(dec)
        if fn is None:
            err("composite %s: no decomposition @%s" % (name, dec))
        return run_func(module, f, fn, args)
    err("composite %s: no decomposition" % name)


def run_region(module, f: Faults, env, known, block, args, arg_known):
    """Lower.lean:503-519: run a block whose arguments are `args`, seeing the
    enclosing values; returns its results and which of them are known integer
    scalars."""
    env = dict(env)
    known = dict(known)
    for (n, _), a, k in zip(block.args, args, arg_known):
        env[n] = a
        if k is None:
            known.pop(n, None)
        else:
            known[n] = k
    for o in block.ops:
        try:
            xs = [env[nm] for nm in o.operands]
        except KeyError as e:
            raise M.ShloError("undefined value %s" % e)
        rs = run_op(f, o, xs, module, env, known)
        if len(rs) != len(o.results):
            raise M.ShloError("%s: %d results for %d names" % (o.name, len(rs), len(o.results)))
        env.update(zip(o.results, rs))
        if len(o.results) == 1:
            v = const_eval(known, o)
            if v is None:
                known.pop(o.results[0], None)
            else:
                known[o.results[0]] = v
    try:
        outs = [env[nm] for nm in block.ret]
    except KeyError as e:
        raise M.ShloError("undefined value %s" % e)
    return outs, [known.get(nm) for nm in block.ret]


def run_func(module, f: Faults, fn, args):
    """Lower.lean:521-526."""
    if len(args) != len(fn.args):
        raise M.ShloError("@%s takes %d arguments, got %d" % (fn.name, len(fn.args), len(args)))
    return run_region(module, f, {}, {}, fn.body, args, [None] * len(args))[0]
