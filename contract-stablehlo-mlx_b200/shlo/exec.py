"""StablehloMlx/Exec.lean restated, with a reader for the generic form it runs.

`load` parses a module (the generic form `Tests/OpTests.lean:39-97` writes:
one op per line, `"stablehlo.x"(%a, %b) {attrs} : (types) -> type`),
`prepare` wraps `main` as a traced function (Exec.lean:30-31, through
`mlx.compile_`), and `call` runs and evaluates it (Exec.lean:34-37).

The reader carries single-block functions; region ops (`while`, `reduce`) are
refused as not carried by this reader.

Ops run one at a time, as Lower.lean issues them; the fused launches of a
compiled function are chosen below the boundary, by libshlo_cuda's recorder
(csrc/fusion.cu), so this mirror and the unchanged Lean host get the same ones.
"""
from __future__ import annotations

import re
from dataclasses import dataclass, field
from typing import Dict, List

from . import lower as L
from . import mlx as M

_TYPE = re.compile(r"tensor<([^>]*)>")


def parse_ty(s: str) -> L.Ty:
    m = _TYPE.fullmatch(s.strip())
    if not m:
        raise M.ShloError("type %s is not carried" % s)
    parts = m.group(1).split("x")
    dims = tuple(int(p) for p in parts[:-1])
    return L.Ty(dims, parts[-1])


def split_top(s: str, sep: str = ",") -> List[str]:
    """Split at `sep` outside (), [], {}, <> and quotes."""
    out, depth, cur, q = [], 0, [], False
    for ch in s:
        if ch == '"':
            q = not q
        elif not q and ch in "([{<":
            depth += 1
        elif not q and ch in ")]}>":
            depth -= 1
        if ch == sep and depth == 0 and not q:
            out.append("".join(cur))
            cur = []
        else:
            cur.append(ch)
    if "".join(cur).strip():
        out.append("".join(cur))
    return out


def _types_of(s: str) -> List[L.Ty]:
    s = s.strip()
    if s.startswith("(") and s.endswith(")"):
        s = s[1:-1]
    return [parse_ty(t) for t in split_top(s) if t.strip()]


@dataclass
class Func:
    name: str
    args: List[tuple]         # (name, Ty)
    ops: List[L.Op]
    ret: List[str]


@dataclass
class Module:
    funcs: Dict[str, Func] = field(default_factory=dict)

    def run_func(self, f: L.Faults, fn: Func, args: List[M.Arr]) -> List[M.Arr]:
        """Lower.lean:521-526 (one block, no trace-time scalars)."""
        if len(args) != len(fn.args):
            raise M.ShloError("@%s takes %d arguments, got %d" % (fn.name, len(fn.args), len(args)))
        env = {n: a for (n, _), a in zip(fn.args, args)}
        for o in fn.ops:
            try:
                xs = [env[n] for n in o.operands]
            except KeyError as e:
                raise M.ShloError("undefined value %s" % e)
            rs = L.run_op(f, o, xs, self)
            if len(rs) != len(o.results):
                raise M.ShloError("%s: %d results for %d names" % (o.name, len(rs), len(o.results)))
            env.update(zip(o.results, rs))
        return [env[n] for n in fn.ret]


_OP = re.compile(r'^(%[\w#:]+(?:\s*,\s*%[\w#]+)*)\s*=\s*"([\w.]+)"\((.*?)\)\s*(\{.*\})?\s*:\s*(\(.*\))\s*->\s*(.+)$')
_FUNC = re.compile(r"^func\.func\s+(?:public\s+|private\s+)?@(\w+)\((.*)\)\s*->\s*(.*)\{$")


def parse(text: str) -> Module:
    mod = Module()
    cur = None
    for raw in text.splitlines():
        line = raw.strip()
        if line == "}":
            cur = None
            continue
        if not line or line.startswith("//") or line.startswith("module"):
            continue
        fm = _FUNC.match(line)
        if fm:
            args = []
            for a in split_top(fm.group(2)):
                nm, ty = a.split(":", 1)
                args.append((nm.strip(), parse_ty(ty)))
            cur = Func(fm.group(1), args, [], None)
            mod.funcs[cur.name] = cur
            continue
        if cur is None:
            raise M.ShloError("unexpected line outside a function: %s" % line)
        if line.startswith("func.return") or line.startswith('"func.return"'):
            body = line.split("func.return", 1)[1].split(":")[0]
            cur.ret = [t.strip() for t in body.split(",") if t.strip()]
            continue
        om = _OP.match(line)
        if not om:
            raise M.ShloError("op not carried by this reader: %s" % line[:120])
        res = [r.strip() for r in om.group(1).split(",")]
        operands = [x.strip() for x in split_top(om.group(3))] if om.group(3).strip() else []
        attrs = {}
        if om.group(4):
            for kv in split_top(om.group(4).strip()[1:-1]):
                if "=" in kv:
                    k, v = kv.split("=", 1)
                    attrs[k.strip()] = v.strip()
        in_tys = _types_of(om.group(5))
        out_tys = _types_of(om.group(6))
        cur.ops.append(L.Op(om.group(2), operands, res, attrs, in_tys, out_tys))
    return mod


@dataclass
class Loaded:
    module: Module
    main: Func


def load(text: str) -> Loaded:
    m = parse(text)
    if "main" not in m.funcs:
        raise M.ShloError("the module has no @main")
    return Loaded(m, m.funcs["main"])


def prepare(l: Loaded, faults: L.Faults = None, compile: bool = True) -> M.Fn:
    faults = faults or L.Faults()
    return M.compile_(lambda args: l.module.run_func(faults, l.main, args), compile)


def call(fn: M.Fn, inputs: List[M.Arr]) -> List[M.Arr]:
    outs = M.apply(fn, inputs)
    M.eval_(outs)
    return outs


def arg_tys(l: Loaded) -> List[L.Ty]:
    return [t for _, t in l.main.args]


def arr_of_bytes(t: L.Ty, b: bytes) -> M.Arr:
    return M.of_bytes(b, list(t.dims), L.el_dtype(t.el))
