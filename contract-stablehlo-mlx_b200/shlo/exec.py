"""StablehloMlx/Exec.lean restated.

`load` reads a module (shlo.parse, the restatement of Parse.lean: the generic
form with regions for `while`, `reduce` and composite bodies), `prepare` wraps
`main` as a traced function (Exec.lean:30-31, through `mlx.compile_`), and
`call` runs and evaluates it (Exec.lean:34-37). The function body runs through
shlo.lower's `run_func` (Lower.lean:503-526): ops one at a time, regions with
the enclosing values in scope, `while` unrolled at trace time.

The fused launches of a compiled function are chosen below the boundary, by
libshlo_cuda's recorder (csrc/fusion.cu), so this mirror and the unchanged
Lean host get the same ones.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List

from . import lower as L
from . import mlx as M
from . import parse as P


@dataclass
class Module:
    funcs: Dict[str, P.FuncDef] = field(default_factory=dict)

    def func(self, name: str):
        return self.funcs.get(name)


def parse(text: str) -> Module:
    try:
        fs = P.parse(text)
    except P.ParseError as e:
        raise M.ShloError(str(e))
    return Module({fn.name: fn for fn in fs})


@dataclass
class Loaded:
    module: Module
    main: P.FuncDef


def load(text: str) -> Loaded:
    """Exec.lean:21-27."""
    m = parse(text)
    if "main" not in m.funcs:
        raise M.ShloError("the module has no @main")
    return Loaded(m, m.funcs["main"])


def prepare(l: Loaded, faults: L.Faults = None, compile: bool = True) -> M.Fn:
    """Exec.lean:30-31."""
    faults = faults or L.Faults()
    return M.compile_(lambda args: L.run_func(l.module, faults, l.main, args), compile)


def call(fn: M.Fn, inputs: List[M.Arr]) -> List[M.Arr]:
    """Exec.lean:34-37."""
    outs = M.apply(fn, inputs)
    M.eval_(outs)
    return outs


def arg_tys(l: Loaded) -> List[L.Ty]:
    return [t for _, t in l.main.args]


def arr_of_bytes(t: L.Ty, b: bytes) -> M.Arr:
    """Exec.lean:42-43."""
    return M.of_bytes(b, list(t.dims), L.el_dtype(t.el))
