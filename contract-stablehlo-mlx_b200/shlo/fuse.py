"""Bit-preserving fusions for the executor (an optimisation of Lower.lean's
one-op-at-a-time lowering; the reference has none).

Three patterns of the denoiser and encoder modules are run as one launch each,
when nothing else reads the intermediate values:

  * dense: dot_general (no batching dimensions, one free dimension on the
    right) -> add with a broadcast 1-D bias over the last dimension
    [-> add with a residual of the output's type that is already computed]:
    `shlo_mul_mat_bias`, whose epilogue runs the same binary32 adds, rounded
    one at a time, in the module's operand order;
  * layer norm: ggml.norm -> multiply by a broadcast 1-D gain -> add a
    broadcast 1-D bias: `shlo_norm_affine`;
  * attention of one head width 64 over 128 or 256 positions: dot_general
    (q k^T, batching over batch and head) -> ggml.soft_max -> dot_general
    (p v) -> transpose to [batch, position, head, width]: `shlo_attention`,
    which reads q, k and v where they lie (strided views of the projection)
    and writes the transposed layout.

Every rounding of the unfused sequence is kept, so the results are the same
bits (tests/test_gpu_fuse.py checks whole modules fused against unfused). The
planted faults change what ops mean, so a run with any fault set is not fused.
"""
from __future__ import annotations

from dataclasses import dataclass, fields
from typing import Dict, List, Optional

from . import lower as L
from . import mlx as M
from . import run as Run


@dataclass
class Fused:
    kind: str                 # "dense", "norm" or "attention"
    result: str               # the value the last fused op defines
    skip: List[int]           # op indices replaced by this one
    bias: str = ""
    gain: str = ""
    res: str = ""
    flags: int = 0
    v: str = ""               # attention: the value operand
    scale: int = 0            # attention: the soft_max scale (binary32 bits)


def any_fault(f: L.Faults) -> bool:
    return any(getattr(f, fl.name) for fl in fields(f))


def _bcast_last_1d(op: L.Op) -> bool:
    """broadcast_in_dim of a 1-D value onto the last dimension of its output."""
    if op.name != "stablehlo.broadcast_in_dim" or len(op.in_tys) != 1 or len(op.in_tys[0].dims) != 1:
        return False
    mp = L.ints(op.attr("broadcast_dimensions") or "")
    out = op.out_tys[0]
    return mp == [len(out.dims) - 1] and op.in_tys[0].dims[0] == out.dims[-1]


def _ggml(op: L.Op) -> str:
    """The ggml.* routine a custom_call or composite names, else ""."""
    if op.name not in ("stablehlo.custom_call", "stablehlo.composite"):
        return ""
    return (op.attr("name") or op.attr("call_target_name") or "").replace('"', "")


def _dims(dn: str, key: str) -> List[int]:
    return L.ints(L.field_(dn, key))


def _attention(ops: List[L.Op], i: int, single_user, ready_before) -> Optional[Fused]:
    """The attention chain whose scores dot_general is ops[i], if it matches."""
    o = ops[i]
    dn = o.attr("dot_dimension_numbers") or ""
    if (_dims(dn, "lhs_batching_dimensions") != [0, 2] or _dims(dn, "rhs_batching_dimensions") != [0, 2]
            or _dims(dn, "lhs_contracting_dimensions") != [3] or _dims(dn, "rhs_contracting_dimensions") != [3]):
        return None
    tq, tk = o.in_tys
    if tq.el != "f32" or tk.el != "f32" or len(tq.dims) != 4 or list(tq.dims) != list(tk.dims):
        return None
    B, S, H, W = tq.dims
    if W != 64 or S not in (128, 256) or list(o.out_tys[0].dims) != [B, H, S, S]:
        return None
    j = single_user(o.results[0])
    if j is None or _ggml(ops[j]) != "ggml.soft_max" or ops[j].operands[0] != o.results[0]:
        return None
    attrs = ops[j].attr("composite_attributes") or ops[j].attr("backend_config") or ""
    l = single_user(ops[j].results[0])
    if l is None or ops[l].name != "stablehlo.dot_general" or ops[l].operands[0] != ops[j].results[0]:
        return None
    dn2 = ops[l].attr("dot_dimension_numbers") or ""
    if (_dims(dn2, "lhs_batching_dimensions") != [0, 1] or _dims(dn2, "rhs_batching_dimensions") != [0, 2]
            or _dims(dn2, "lhs_contracting_dimensions") != [3] or _dims(dn2, "rhs_contracting_dimensions") != [1]):
        return None
    v = ops[l].operands[1]
    if list(ops[l].in_tys[1].dims) != [B, S, H, W] or ops[l].in_tys[1].el != "f32" or not ready_before(v, i):
        return None
    t = single_user(ops[l].results[0])
    if (t is None or ops[t].name != "stablehlo.transpose"
            or L.ints(ops[t].attr("permutation") or "") != [0, 2, 1, 3] or list(ops[t].out_tys[0].dims) != [B, S, H, W]):
        return None
    return Fused("attention", ops[t].results[0], [j, l, t], v=v, scale=L.f32_attr(attrs, "scale"))


def plan(fn) -> Dict[int, Fused]:
    """Fusions of one function body, keyed by the index of the op that runs
    the fused launch (the dot_general or the norm)."""
    ops: List[L.Op] = fn.ops
    uses: Dict[str, int] = {}
    user: Dict[str, int] = {}
    producer: Dict[str, int] = {}
    for i, o in enumerate(ops):
        for r in o.results:
            producer[r] = i
        for a in o.operands:
            uses[a] = uses.get(a, 0) + 1
            user[a] = i
    for r in fn.ret or []:
        uses[r] = uses.get(r, 0) + 1

    def single_user(v: str) -> Optional[int]:
        return user.get(v) if uses.get(v, 0) == 1 else None

    def ready_before(v: str, i: int) -> bool:
        return v not in producer or producer[v] < i

    def other(o: L.Op, v: str):
        a, b = o.operands
        return (b, False) if a == v else (a, True)  # (the other operand, is it the left one)

    out: Dict[int, Fused] = {}
    taken = set()
    for i, o in enumerate(ops):
        if o.name == "stablehlo.dot_general" and o.out_tys and o.out_tys[0].el == "f32":
            dn = o.attr("dot_dimension_numbers") or ""
            if L.ints(L.field_(dn, "lhs_batching_dimensions")) or L.ints(L.field_(dn, "rhs_batching_dimensions")):
                fz = _attention(ops, i, single_user, ready_before)
                if fz is not None and not taken.intersection(fz.skip):
                    out[i] = fz
                    taken.update(fz.skip)
                continue
            if len(o.in_tys[1].dims) != 2:
                continue
            j = single_user(o.results[0])
            if j is None or ops[j].name != "stablehlo.add" or j in taken:
                continue
            bb, bb_left = other(ops[j], o.results[0])
            k = producer.get(bb)
            if k is None or single_user(bb) != j or not _bcast_last_1d(ops[k]) or not ready_before(ops[k].operands[0], i):
                continue
            fz = Fused("dense", ops[j].results[0], [j, k], bias=ops[k].operands[0],
                       flags=Run.EP_BIAS | (Run.EP_BIAS_LHS if bb_left else 0))
            l = single_user(ops[j].results[0])
            if l is not None and ops[l].name == "stablehlo.add" and l not in taken:
                h, h_left = other(ops[l], ops[j].results[0])
                if ready_before(h, i) and ops[l].out_tys[0].dims == o.out_tys[0].dims and h != ops[j].results[0]:
                    fz.res, fz.result = h, ops[l].results[0]
                    fz.skip.append(l)
                    fz.flags |= Run.EP_RES | (Run.EP_RES_LHS if h_left else 0)
            out[i] = fz
            taken.update(fz.skip)
        elif o.name == "stablehlo.custom_call" and (o.attr("call_target_name") or "").replace('"', "") == "ggml.norm":
            j = single_user(o.results[0])
            if j is None or ops[j].name != "stablehlo.multiply" or ops[j].operands[0] != o.results[0]:
                continue
            gg = ops[j].operands[1]
            kg = producer.get(gg)
            if kg is None or single_user(gg) != j or not _bcast_last_1d(ops[kg]) or not ready_before(ops[kg].operands[0], i):
                continue
            l = single_user(ops[j].results[0])
            if l is None or ops[l].name != "stablehlo.add" or ops[l].operands[0] != ops[j].results[0]:
                continue
            bb = ops[l].operands[1]
            kb = producer.get(bb)
            if kb is None or single_user(bb) != l or not _bcast_last_1d(ops[kb]) or not ready_before(ops[kb].operands[0], i):
                continue
            out[i] = Fused("norm", ops[l].results[0], [j, kg, l, kb], bias=ops[kb].operands[0],
                           gain=ops[kg].operands[0])
            taken.update(out[i].skip)
    return out


def run_fused(fz: Fused, o: L.Op, env: Dict[str, M.Arr]) -> M.Arr:
    out = o.out_tys[0]
    if fz.kind == "attention":
        B, S, H, W = o.in_tys[0].dims
        y = Run.attention(env[o.operands[0]], env[o.operands[1]], env[fz.v], B, S, H, W, fz.scale)
        return M.reshape(y, [B, S, H, W])
    if fz.kind == "dense":
        dn = o.attr("dot_dimension_numbers") or ""
        lc = L.ints(L.field_(dn, "lhs_contracting_dimensions"))[0]
        rc = L.ints(L.field_(dn, "rhs_contracting_dimensions"))[0]
        ta, tb = o.in_tys
        lf = [d for d in range(len(ta.dims)) if d != lc]
        rf = [d for d in range(len(tb.dims)) if d != rc]
        K, Mm = ta.dims[lc], tb.dims[rf[0]]
        N = out.count // Mm
        a2 = M.reshape(M.transpose(env[o.operands[0]], lf + [lc]), [N, K])
        b2 = M.reshape(M.transpose(env[o.operands[1]], rf + [rc]), [Mm, K])
        res = M.reshape(env[fz.res], [N * Mm]) if fz.res else None
        y = Run.mul_mat_bias(b2, a2, K, Mm, N, N, 0, env[fz.bias], res, fz.flags)
        return M.reshape(y, list(out.dims))
    rows, cols = L.rows_cols(out)
    attrs = o.attr("backend_config") or ""
    y = Run.norm_affine(env[o.operands[0]], cols, rows, L.f32_attr(attrs, "eps"), env[fz.gain], env[fz.bias])
    return M.reshape(y, list(out.dims))
