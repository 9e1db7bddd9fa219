"""The reader (shlo/parse.py, StablehloMlx/Parse.lean restated) on the
generic path's region ops, and the lowering's trace-time scalars (Lower.lean's
constEval) -- no GPU needed: nothing here runs a device op."""
import pytest

import generic_modules as GM
from shlo import exec as E
from shlo import lower as L
from shlo import mlx as M


def test_while_reads_its_two_regions():
    l = E.load(GM.while_accumulate(8, 3))
    (c0, w) = l.main.ops
    assert w.name == "stablehlo.while" and w.results == ["%r#0", "%r#1"] and w.operands == ["%c0", "%x"]
    cond, body = w.regions
    assert [a for a, _ in cond.args] == ["%i", "%acc"] and cond.args[0][1].el == "i64"
    assert [o.name for o in cond.ops] == ["stablehlo.constant", "stablehlo.compare"] and cond.ret == ["%c"]
    assert body.ret == ["%i2", "%a2"]
    assert l.main.ret == ["%r#1"]
    assert w.out_tys[1].dims == (8,)


def test_reduce_gather_dynamic_slice_read():
    r = E.load(GM.reduce_max(4, 8, [1])).main.ops[0]
    assert r.name == "stablehlo.reduce" and L.ints(r.attr("dimensions")) == [1]
    assert r.regions[0].ops[0].name == "stablehlo.maximum"
    g = E.load(GM.gather1d(16, 8)).main.ops[0]
    assert L.field_(g.attr("dimension_numbers"), "collapsed_slice_dims") == "[0]"
    assert L.ints(g.attr("slice_sizes")) == [1]
    d = E.load(GM.dynamic_slice(16, 8, (2, 3, 1), (4, 4))).main.ops[-1]
    assert d.name == "stablehlo.dynamic_slice" and L.ints(d.attr("slice_sizes")) == [4, 4]


def test_const_eval_follows_trace_time_arithmetic():
    ops = E.load(GM.dynamic_slice(16, 8, (2, 3, 1), (4, 4))).main.ops
    known = {}
    for o in ops[:-1]:
        v = L.const_eval(known, o)
        if v is not None:
            known[o.results[0]] = v
    assert known == {"%a": 2, "%b": 3, "%s0": 5, "%s1": 1}
    cond = E.load(GM.while_accumulate(8, 3)).main.ops[1].regions[0]
    k = {"%i": 2}
    for o in cond.ops:
        v = L.const_eval(k, o)
        if v is not None:
            k[o.results[0]] = v
    assert k["%c"] == 1  # 2 < 3


def test_parse_errors_are_reported():
    with pytest.raises(M.ShloError, match="parse error"):
        E.load('module { func.func @main(%x: tensor<4xf32>) -> tensor<4xf32> { %y = stablehlo.add %x, %x } }')
