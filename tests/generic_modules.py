"""Modules of the generic path (contract-ggml-stablehlo's form: region ops,
binary64 as uint64 bit patterns, trace-time scalars) for the reader and the
lowering of StablehloMlx/Parse.lean and Lower.lean:317-470 -- test
infrastructure. Each builder returns module text; the tests run it and compare
with numpy."""
from __future__ import annotations


def T(*dims, el="f32") -> str:
    return "tensor<" + "".join("%dx" % d for d in dims) + el + ">"


def while_accumulate(n: int, trips: int, el: str = "f32", cond_from_data: bool = False) -> str:
    """acc = x; for i in [0, trips): acc = acc + y  -- the loop counter and bound
    are trace-time scalars (or, with cond_from_data, the bound is an argument)."""
    v = T(n, el=el)
    i64 = "tensor<i64>"
    bound = ('    %%n = "stablehlo.constant"() {value = dense<%d> : tensor<i64>} : () -> tensor<i64>\n' % trips
             if not cond_from_data else "")
    nref = "%n" if not cond_from_data else "%lim"
    extra_arg = ", %%lim: %s" % i64 if cond_from_data else ""
    return f"""module {{
  func.func public @main(%x: {v}, %y: {v}{extra_arg}) -> ({v}) {{
    %c0 = "stablehlo.constant"() {{value = dense<0> : tensor<i64>}} : () -> tensor<i64>
    %r:2 = "stablehlo.while"(%c0, %x) ({{
    ^bb0(%i: tensor<i64>, %acc: {v}):
{bound}      %c = "stablehlo.compare"(%i, {nref}) {{comparison_direction = #stablehlo<comparison_direction LT>}} : (tensor<i64>, tensor<i64>) -> tensor<i1>
      "stablehlo.return"(%c) : (tensor<i1>) -> ()
    }}, {{
    ^bb0(%i: tensor<i64>, %acc: {v}):
      %one = "stablehlo.constant"() {{value = dense<1> : tensor<i64>}} : () -> tensor<i64>
      %i2 = "stablehlo.add"(%i, %one) : (tensor<i64>, tensor<i64>) -> tensor<i64>
      %a2 = "stablehlo.add"(%acc, %y) : ({v}, {v}) -> {v}
      "stablehlo.return"(%i2, %a2) : (tensor<i64>, {v}) -> ()
    }}) : (tensor<i64>, {v}) -> (tensor<i64>, {v})
    func.return %r#1 : {v}
  }}
}}
"""


def dynamic_slice(rows: int, cols: int, start_expr, size: tuple, from_data: bool = False) -> str:
    """out = x[s0 : s0 + size0, s1 : s1 + size1] with s0 = a + b (trace-time
    constants) and s1 = the constant start_expr[2] (or an argument, from_data)."""
    a, b, c = start_expr
    src, out = T(rows, cols), T(*size)
    s1 = ('    %%s1 = "stablehlo.constant"() {value = dense<%d> : tensor<i64>} : () -> tensor<i64>\n' % c
          if not from_data else "")
    arg = ", %s1: tensor<i64>" if from_data else ""
    return f"""module {{
  func.func public @main(%x: {src}{arg}) -> ({out}) {{
    %a = "stablehlo.constant"() {{value = dense<{a}> : tensor<i64>}} : () -> tensor<i64>
    %b = "stablehlo.constant"() {{value = dense<{b}> : tensor<i64>}} : () -> tensor<i64>
    %s0 = "stablehlo.add"(%a, %b) : (tensor<i64>, tensor<i64>) -> tensor<i64>
{s1}    %y = "stablehlo.dynamic_slice"(%x, %s0, %s1) {{slice_sizes = array<i64: {size[0]}, {size[1]}>}} : ({src}, tensor<i64>, tensor<i64>) -> {out}
    func.return %y : {out}
  }}
}}
"""


def gather1d(table: int, count: int, table_rank2: bool = False) -> str:
    """out[i] = table[clamp(idx[i], 0, table - 1)] (contract-ggml-stablehlo's gather1d)."""
    tt = T(table, 1) if table_rank2 else T(table)
    it, out = T(count, el="i64"), T(count)
    return f"""module {{
  func.func public @main(%t: {tt}, %idx: {it}) -> ({out}) {{
    %g = "stablehlo.gather"(%t, %idx) {{dimension_numbers = #stablehlo.gather<offset_dims = [], collapsed_slice_dims = [0], start_index_map = [0], index_vector_dim = 1>, indices_are_sorted = false, slice_sizes = array<i64: 1>}} : ({tt}, {it}) -> {out}
    func.return %g : {out}
  }}
}}
"""


def reduce_max(rows: int, cols: int, dims, body: str = "stablehlo.maximum") -> str:
    """out = max(init, max over `dims` of x)."""
    src = T(rows, cols)
    keep = [d for d in (rows, cols)]
    out_dims = [n for i, n in enumerate(keep) if i not in dims]
    out = T(*out_dims)
    ds = ", ".join(str(d) for d in dims)
    return f"""module {{
  func.func public @main(%x: {src}, %init: tensor<f32>) -> ({out}) {{
    %r = "stablehlo.reduce"(%x, %init) ({{
    ^bb0(%p: tensor<f32>, %q: tensor<f32>):
      %m = "{body}"(%p, %q) : (tensor<f32>, tensor<f32>) -> tensor<f32>
      "stablehlo.return"(%m) : (tensor<f32>) -> ()
    }}) {{dimensions = array<i64: {ds}>}} : ({src}, tensor<f32>) -> {out}
    func.return %r : {out}
  }}
}}
"""
