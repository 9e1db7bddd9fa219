"""The fused launches against the unfused sequences they replace, bit for bit.

The fusions are chosen below the boundary, by the recorder of compiled
functions (csrc/fusion.cu): a compiled call (shlo_compile with enable = 1)
runs the fused kernels, an uncompiled call runs the ops one at a time as
Lower.lean issues them. Checked here: the fused kernels alone on random data
with specials; whole modules (the encoder layer, the denoiser, the attention
block) compiled against uncompiled, with the number of fused chains the
recorder reports; the feed-forward block's two products, the first writing
its result in the second's packed operand layout; chains it must leave alone
(an intermediate read elsewhere, a planted fault); and a traced function whose
capture call departs from its eager call, which must run unfused with the
eager result."""
from __future__ import annotations

import re

import numpy as np
import pytest

from shlo import denoiser as D
from shlo import exec as E
from shlo import lower as L
from shlo import mlx as M
from shlo import run as Run

pytestmark = pytest.mark.gpu


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


@pytest.fixture(autouse=True)
def _pinned():
    M.set_flavor("pinned")
    yield


def specials(rng, shape):
    a = rng.standard_normal(shape).astype(np.float32)
    flat = a.reshape(-1)
    idx = rng.choice(flat.size, size=max(1, flat.size // 50), replace=False)
    flat[idx] = rng.choice(np.array([np.inf, -np.inf, np.nan, 0.0, -0.0, 1e-40, -3e38], np.float32), idx.size)
    return a


@pytest.mark.parametrize("K,Mm,R", [(512, 1536, 300), (64, 256, 256), (196, 130, 50), (737, 64, 70), (16, 8, 5),
                                    (2048, 512, 129), (256, 64, 512)])
@pytest.mark.parametrize("flags", [Run.EP_BIAS, Run.EP_BIAS | Run.EP_BIAS_LHS,
                                   Run.EP_BIAS | Run.EP_RES | Run.EP_RES_LHS, Run.EP_BIAS | Run.EP_BIAS_LHS | Run.EP_RES])
def test_mul_mat_bias_matches_unfused(K, Mm, R, flags):
    rng = np.random.default_rng(K * 31 + Mm + R + flags)
    w = M.of_numpy(specials(rng, (Mm, K)) * np.float32(0.1))
    x = M.of_numpy(specials(rng, (R, K)))
    b = M.of_numpy(specials(rng, (Mm,)))
    h = M.of_numpy(specials(rng, (R, Mm)))
    y = M.reshape(Run.mul_mat(w, x, K, Mm, R, R, 0), [R, Mm])
    bb = M.broadcast(M.reshape(b, [1, Mm]), [R, Mm])
    z = M.binary(M.opAdd, bb, y) if flags & Run.EP_BIAS_LHS else M.binary(M.opAdd, y, bb)
    if flags & Run.EP_RES:
        z = M.binary(M.opAdd, h, z) if flags & Run.EP_RES_LHS else M.binary(M.opAdd, z, h)
    want = M.to_numpy(z)
    got = M.to_numpy(Run.mul_mat_bias(w, x, K, Mm, R, R, 0, b, M.reshape(h, [R * Mm]) if flags & Run.EP_RES else None,
                                      flags))
    assert np.array_equal(bits(got).reshape(-1), bits(want).reshape(-1))


@pytest.mark.parametrize("K,Mm,R,split", [
    (512, 2048, 1100, None),   # k_mul_mat_tm, whole stages a segment, a partial last row tile
    (600, 1024, 2100, None),   # the fold after groups of 4 k, and a K tail of 8
    (512, 1002, 2200, None),   # a partial column tile, M not a multiple of 4 (element stores)
    (512, 2048, 1100, "2"),    # halves of the fold tree: the last CTA of a tile runs the epilogue
    (512, 64, 40000, None),    # one warp along m: the product, then the gelu_erf kernel
    (512, 1536, 300, None),    # a small product (k_mul_mat_seg): the same
])
@pytest.mark.parametrize("flags", [Run.EP_BIAS, Run.EP_BIAS | Run.EP_BIAS_LHS | Run.EP_RES])
def test_mul_mat_bias_gelu_matches_unfused(K, Mm, R, split, flags, monkeypatch):
    """The dense chain with gelu_erf in the product's epilogue (FFN1's form)
    against the product, the adds and the gelu_erf kernel, bit for bit."""
    if split:
        monkeypatch.setenv("SHLO_MM_SPLIT", split)
    rng = np.random.default_rng(K + Mm * 3 + R + flags)
    w = M.of_numpy(specials(rng, (Mm, K)) * np.float32(0.05))
    x = M.of_numpy(specials(rng, (R, K)))
    b = M.of_numpy(specials(rng, (Mm,)))
    h = M.of_numpy(specials(rng, (R, Mm)))
    y = M.reshape(Run.mul_mat(w, x, K, Mm, R, R, 0), [R, Mm])
    bb = M.broadcast(M.reshape(b, [1, Mm]), [R, Mm])
    z = M.binary(M.opAdd, bb, y) if flags & Run.EP_BIAS_LHS else M.binary(M.opAdd, y, bb)
    if flags & Run.EP_RES:
        z = M.binary(M.opAdd, h, z) if flags & Run.EP_RES_LHS else M.binary(M.opAdd, z, h)
    want = M.to_numpy(Run.gelu_erf(M.reshape(z, [R * Mm]), R * Mm))
    got = M.to_numpy(Run.mul_mat_bias(w, x, K, Mm, R, R, 0, b, M.reshape(h, [R * Mm]) if flags & Run.EP_RES else None,
                                      flags | Run.EP_GELU))
    assert np.array_equal(bits(got).reshape(-1), bits(want).reshape(-1))


def test_mul_mat_bias_gelu_refused_stock():
    M.set_flavor("stock")
    try:
        w = M.of_numpy(np.ones((256, 64), np.float32))
        x = M.of_numpy(np.ones((300, 64), np.float32))
        b = M.of_numpy(np.zeros(256, np.float32))
        with pytest.raises(M.ShloError, match="not carried"):
            M.to_numpy(Run.mul_mat_bias(w, x, 64, 256, 300, 300, 0, b, None, Run.EP_BIAS | Run.EP_GELU))
    finally:
        M.set_flavor("pinned")


@pytest.mark.parametrize("cols,rows", [(512, 300), (1024, 17), (36, 9), (1100, 5), (13, 4)])
def test_norm_affine_matches_unfused(cols, rows):
    rng = np.random.default_rng(cols + rows)
    x = M.of_numpy(specials(rng, (rows, cols)))
    g = M.of_numpy(specials(rng, (cols,)))
    b = M.of_numpy(specials(rng, (cols,)))
    n = M.reshape(Run.norm(x, cols, rows, 0x3727C5AC), [rows, cols])
    t = M.binary(M.opMul, n, M.broadcast(M.reshape(g, [1, cols]), [rows, cols]))
    want = M.to_numpy(M.binary(M.opAdd, t, M.broadcast(M.reshape(b, [1, cols]), [rows, cols])))
    got = M.to_numpy(Run.norm_affine(x, cols, rows, 0x3727C5AC, g, b))
    assert np.array_equal(bits(got).reshape(-1), bits(want).reshape(-1))


def run_counted(capfd, monkeypatch, fn, args):
    """Call a compiled function once (recording it) and return its output and
    the fused chains the recorder reported."""
    monkeypatch.setenv("SHLO_GRAPH_VERBOSE", "1")
    capfd.readouterr()
    out = M.to_numpy(E.call(fn, args)[0])
    err = capfd.readouterr().err
    monkeypatch.delenv("SHLO_GRAPH_VERBOSE")
    m = re.search(r"recorded: (\d+) launches, (\d+) fused chains", err)
    return out, (int(m.group(2)) if m else None), err


@pytest.mark.parametrize("cfg,B", [(D.ENCODER, 2), (D.Config(layers=2), 3)])
def test_modules_fused_equal_unfused(cfg, B, capfd, monkeypatch):
    w = D.init_weights(cfg, seed=9)
    W = [M.of_numpy(w[n]) for n, _ in D.weight_specs(cfg)]
    X = [M.of_numpy(a) for a in D.inputs(cfg, B, seed=4)]
    l = E.load(D.module_text(cfg, B))
    want = M.to_numpy(E.call(E.prepare(l, None, False), X + W)[0])
    fn = E.prepare(l, None, True)
    got, chains, err = run_counted(capfd, monkeypatch, fn, X + W)
    # per layer: qkv, output (+ residual), ffn1, ffn2 (+ residual) dense chains, two
    # layer norms, and the attention block where the fused kernel carries its
    # positions (128 or 256: not the encoder's 196); two timestep dense chains
    per_layer = 6 + (1 if cfg.seq in (128, 256) else 0)
    assert chains == per_layer * cfg.layers + (2 if cfg.timestep else 0), err
    # packed handoffs a layer: norm -> QKV, norm -> FFN1, FFN1 -> FFN2, and
    # attention -> output projection where the attention is fused
    m = re.search(r"handing a packed operand on: (\d+)", err)
    assert m and int(m.group(1)) == (3 + (1 if cfg.seq in (128, 256) else 0)) * cfg.layers, err
    assert np.array_equal(bits(got), bits(want))
    again = M.to_numpy(E.call(fn, X + W)[0])  # the replay
    assert np.array_equal(bits(again), bits(want))


def ffn_text(R, K1, F, D2, residual):
    """x [R, K1] -> dense (w1 [F, K1], b1) -> gelu_erf -> dense (w2 [D2, F], b2)
    [-> + r], the feed-forward block's chain of two dense products."""
    T = lambda *d: "tensor<" + "".join("%dx" % x for x in d) + "f32>"
    dn = ('{dot_dimension_numbers = #stablehlo.dot<lhs_contracting_dimensions = [1], '
          'rhs_contracting_dimensions = [1]>}')
    res_arg = ", %%r: %s" % T(R, D2) if residual else ""
    tail = ('    %%o = "stablehlo.add"(%%r, %%z2) : (%s, %s) -> %s\n    func.return %%o : %s\n'
            % (T(R, D2), T(R, D2), T(R, D2), T(R, D2)) if residual else "    func.return %%z2 : %s\n" % T(R, D2))
    return f"""module {{
  func.func public @main(%x: {T(R, K1)}, %w1: {T(F, K1)}, %b1: {T(F)}, %w2: {T(D2, F)}, %b2: {T(D2)}{res_arg}) -> {T(R, D2)} {{
    %y1 = "stablehlo.dot_general"(%x, %w1) {dn} : ({T(R, K1)}, {T(F, K1)}) -> {T(R, F)}
    %c1 = "stablehlo.broadcast_in_dim"(%b1) {{broadcast_dimensions = array<i64: 1>}} : ({T(F)}) -> {T(R, F)}
    %z1 = "stablehlo.add"(%y1, %c1) : ({T(R, F)}, {T(R, F)}) -> {T(R, F)}
    %g = "stablehlo.custom_call"(%z1) {{call_target_name = "ggml.gelu_erf", backend_config = ""}} : ({T(R, F)}) -> {T(R, F)}
    %y2 = "stablehlo.dot_general"(%g, %w2) {dn} : ({T(R, F)}, {T(D2, F)}) -> {T(R, D2)}
    %c2 = "stablehlo.broadcast_in_dim"(%b2) {{broadcast_dimensions = array<i64: 1>}} : ({T(D2)}) -> {T(R, D2)}
    %z2 = "stablehlo.add"(%y2, %c2) : ({T(R, D2)}, {T(R, D2)}) -> {T(R, D2)}
{tail}  }}
}}
"""


@pytest.mark.parametrize("R,K1,F,D2,split,linked", [
    (1100, 512, 2048, 512, None, True),    # gelu epilogue writes the packed x (a partial last row tile); seg consumer
    (1100, 512, 2048, 2048, None, True),   # both products on k_mul_mat_tm
    (1100, 512, 2048, 512, "2", True),     # halves of the fold tree: the last CTA writes the packed tile
    (4000, 256, 576, 1024, None, True),    # F not a multiple of the 128-column tile
    (4000, 256, 576, 512, None, True),     # the products' padded rows differ: the pack kernel packs it
    (300, 512, 1024, 512, None, True),     # the first product on k_mul_mat_seg: packed by the pack kernel
    (1100, 512, 1000, 512, None, False),   # F not a multiple of 64: no handoff, each packs its own
])
@pytest.mark.parametrize("residual", [False, True])
def test_ffn_packed_handoff_matches_unfused(R, K1, F, D2, split, linked, residual, capfd, monkeypatch):
    """Two dense chains joined by gelu_erf: compiled, the first writes its result
    in the second's packed x layout (the second skips its pack); uncompiled, the
    ops one at a time. Bit for bit, the recording and its replay."""
    if split:
        monkeypatch.setenv("SHLO_MM_SPLIT", split)
    rng = np.random.default_rng(R + K1 + F + D2 + residual)
    args = [specials(rng, (R, K1)), specials(rng, (F, K1)) * np.float32(0.05), specials(rng, (F,)),
            specials(rng, (D2, F)) * np.float32(0.05), specials(rng, (D2,))]
    if residual:
        args.append(specials(rng, (R, D2)))
    args = [M.of_numpy(a) for a in args]
    l = E.load(ffn_text(R, K1, F, D2, residual))
    want = M.to_numpy(E.call(E.prepare(l, None, False), args)[0])
    fn = E.prepare(l, None, True)
    got, chains, err = run_counted(capfd, monkeypatch, fn, args)
    assert chains == 2, err
    assert ("handing a packed operand on: 1" in err) == linked, err
    assert np.array_equal(bits(got), bits(want))
    again = M.to_numpy(E.call(fn, args)[0])
    assert np.array_equal(bits(again), bits(want))


def test_planted_faults_are_not_fused_away(capfd, monkeypatch):
    """A planted wrong lowering changes the ops, so the chain no longer matches
    and the compiled result keeps the fault's bits (differing from the exact ones)."""
    cfg = D.Config(layers=1)
    w = D.init_weights(cfg, seed=2)
    W = [M.of_numpy(w[n]) for n, _ in D.weight_specs(cfg)]
    X = [M.of_numpy(a) for a in D.inputs(cfg, 1, seed=2)]
    l = E.load(D.module_text(cfg, 1))
    exact = M.to_numpy(E.call(E.prepare(l, None, False), X + W)[0])
    for fault in (L.Faults(dotPlain=True), L.Faults(normGpuOps=True), L.Faults(softMaxFloatSum=True),
                  L.Faults(broadcastFirst=True)):
        eager = M.to_numpy(E.call(E.prepare(l, fault, False), X + W)[0])
        got, chains, err = run_counted(capfd, monkeypatch, E.prepare(l, fault, True), X + W)
        assert np.array_equal(bits(got), bits(eager)), fault
        assert not np.array_equal(bits(got), bits(exact)), fault


def test_intermediate_read_elsewhere_is_not_fused(capfd, monkeypatch):
    """The dense chain's product is also a function output: it must be computed
    on its own, so nothing is fused."""
    text = """module {
  func.func public @main(%x: tensor<64x512xf32>, %w: tensor<256x512xf32>, %b: tensor<256xf32>) -> (tensor<64x256xf32>, tensor<64x256xf32>) {
    %y = "stablehlo.dot_general"(%x, %w) {dot_dimension_numbers = #stablehlo.dot<lhs_contracting_dimensions = [1], rhs_contracting_dimensions = [1]>} : (tensor<64x512xf32>, tensor<256x512xf32>) -> tensor<64x256xf32>
    %bb = "stablehlo.broadcast_in_dim"(%b) {broadcast_dimensions = array<i64: 1>} : (tensor<256xf32>) -> tensor<64x256xf32>
    %z = "stablehlo.add"(%y, %bb) : (tensor<64x256xf32>, tensor<64x256xf32>) -> tensor<64x256xf32>
    func.return %z, %y : tensor<64x256xf32>, tensor<64x256xf32>
  }
}
"""
    rng = np.random.default_rng(1)
    args = [M.of_numpy(rng.standard_normal(s).astype(np.float32)) for s in ((64, 512), (256, 512), (256,))]
    l = E.load(text)
    want = [M.to_numpy(a) for a in E.call(E.prepare(l, None, False), args)]
    got, chains, err = run_counted(capfd, monkeypatch, E.prepare(l, None, True), args)
    assert chains == 0, err
    assert np.array_equal(bits(got), bits(want[0]))


def test_capture_call_departing_from_eager_call_runs_unfused(capfd, monkeypatch):
    """The recorder matches the capture call to the eager call op by op; a
    traced function that does something else the second time must not get the
    first call's fused chain: the recording is dropped and the function runs
    eagerly (unfused) from then on, with its own results."""
    rng = np.random.default_rng(3)
    K, Mm, R = 512, 256, 64
    w = M.of_numpy(rng.standard_normal((Mm, K)).astype(np.float32))
    x = M.of_numpy(rng.standard_normal((R, K)).astype(np.float32))
    b = M.of_numpy(rng.standard_normal((Mm,)).astype(np.float32))
    b2 = M.of_numpy(rng.standard_normal((R, Mm)).astype(np.float32))
    calls = [0]

    def f(args):
        calls[0] += 1
        y = M.reshape(Run.mul_mat(args[0], args[1], K, Mm, R, R, 0), [R, Mm])
        other = M.broadcast(M.reshape(args[2], [1, Mm]), [R, Mm]) if calls[0] != 2 else args[3]
        return [M.binary(M.opAdd, y, other)]

    monkeypatch.setenv("SHLO_GRAPH_VERBOSE", "1")
    capfd.readouterr()
    fn = M.compile_(f, True)
    got = M.to_numpy(M.apply(fn, [w, x, b, b2])[0])
    err = capfd.readouterr().err
    monkeypatch.delenv("SHLO_GRAPH_VERBOSE")
    assert "runs eagerly" in err and "fusion" in err, err
    y = M.reshape(Run.mul_mat(w, x, K, Mm, R, R, 0), [R, Mm])
    want = M.to_numpy(M.binary(M.opAdd, y, M.broadcast(M.reshape(b, [1, Mm]), [R, Mm])))
    assert np.array_equal(bits(got), bits(want))


def attn_text(B, S, H, W, scale_bits, merged=True):
    """q k^T -> soft_max -> p v -> transpose, as the encoder layer writes it;
    `merged`: then the reshape to [B, S, H*W] that ends the fused chain."""
    T = lambda *d: "tensor<" + "".join("%dx" % x for x in d) + "f32>"
    q, s_, o, qkv = T(B, S, H, W), T(B, H, S, S), T(B, H, S, W), T(B, S, 3, H, W)
    m = T(B, S, H * W)
    tail = (f'    %r = "stablehlo.reshape"(%t) : ({q}) -> {m}\n    func.return %r : {m}\n' if merged
            else f"    func.return %t : {q}\n")
    sl = T(B, S, 1, H, W)
    parts = []
    for i in range(3):
        parts.append(
            f'    %sl{i} = "stablehlo.slice"(%qkv) {{start_indices = array<i64: 0, 0, {i}, 0, 0>, limit_indices = '
            f'array<i64: {B}, {S}, {i + 1}, {H}, {W}>, strides = array<i64: 1, 1, 1, 1, 1>}} : ({qkv}) -> {sl}\n'
            f'    %x{i} = "stablehlo.reshape"(%sl{i}) : ({sl}) -> {q}\n')
    return f"""module {{
  func.func public @main(%qkv: {qkv}) -> ({m if merged else q}) {{
{''.join(parts)}    %s = "stablehlo.dot_general"(%x0, %x1) {{dot_dimension_numbers = #stablehlo.dot<lhs_batching_dimensions = [0, 2], rhs_batching_dimensions = [0, 2], lhs_contracting_dimensions = [3], rhs_contracting_dimensions = [3]>}} : ({q}, {q}) -> {s_}
    %p = "stablehlo.custom_call"(%s) {{call_target_name = "ggml.soft_max", backend_config = "scale = 0x{scale_bits:08X} : f32"}} : ({s_}) -> {s_}
    %o = "stablehlo.dot_general"(%p, %x2) {{dot_dimension_numbers = #stablehlo.dot<lhs_batching_dimensions = [0, 1], rhs_batching_dimensions = [0, 2], lhs_contracting_dimensions = [3], rhs_contracting_dimensions = [1]>}} : ({s_}, {q}) -> {o}
    %t = "stablehlo.transpose"(%o) {{permutation = array<i64: 0, 2, 1, 3>}} : ({o}) -> {q}
{tail}  }}
}}
"""


@pytest.mark.parametrize("B,S,H,scale,special,amp", [(2, 256, 8, 0x3E000000, False, 4.0), (1, 128, 3, 0x3E000000, True, 4.0),
                                                     (3, 256, 2, 0x3F800000, True, 4.0), (1, 256, 1, 0x41000000, False, 4.0),
                                                     (2, 256, 4, 0x3E000000, False, 0.05), (1, 128, 2, 0x3E000000, False, 0.3),
                                                     (2, 256, 2, 0x3E000000, False, 1.0)])
def test_attention_matches_unfused(B, S, H, scale, special, amp, capfd, monkeypatch):
    # q, k, v as the strided slices of one projection, as in the encoder layer;
    # specials give NaN and infinite score rows (the soft_max's sequential scan);
    # small amplitudes keep every row's exponentials within a few binades (the
    # group sums added in any order), large ones spread them (the serial chain)
    rng = np.random.default_rng(B * 1000 + S + H)
    a = specials(rng, (B, S, 3, H, 64)) if special else rng.standard_normal((B, S, 3, H, 64)).astype(np.float32)
    x = [M.of_numpy(a * np.float32(amp))]
    for merged in (True, False):
        l = E.load(attn_text(B, S, H, 64, scale, merged))
        want = M.to_numpy(E.call(E.prepare(l, None, False), x)[0])
        got, chains, err = run_counted(capfd, monkeypatch, E.prepare(l, None, True), x)
        # without the final reshape the chain has no end to fuse into -- except
        # with one head, where the value product already is the [B, S, H*64] layout
        assert chains == (1 if merged or H == 1 else 0), err
        assert np.array_equal(bits(got), bits(want))


def then_dense(text, R, K, M2, last, last_ty):
    """A module returning `last` ([..., K] of type last_ty) made to return
    dense(last) = last [R, K] @ w [M2, K]^T + b [M2] instead (new arguments %w, %b)."""
    T = lambda *d: "tensor<" + "".join("%dx" % x for x in d) + "f32>"
    dn = ('{dot_dimension_numbers = #stablehlo.dot<lhs_contracting_dimensions = [1], '
          'rhs_contracting_dimensions = [1]>}')
    head, _, _ = text.partition("    func.return %s : %s\n" % (last, last_ty))
    head = head.replace(") -> (%s) {" % last_ty, ", %%w: %s, %%b: %s) -> (%s) {" % (T(M2, K), T(M2), T(R, M2)), 1)
    head = head.replace(") -> %s {" % last_ty, ", %%w: %s, %%b: %s) -> %s {" % (T(M2, K), T(M2), T(R, M2)), 1)
    return head + f"""    %rr = "stablehlo.reshape"({last}) : ({last_ty}) -> {T(R, K)}
    %y9 = "stablehlo.dot_general"(%rr, %w) {dn} : ({T(R, K)}, {T(M2, K)}) -> {T(R, M2)}
    %c9 = "stablehlo.broadcast_in_dim"(%b) {{broadcast_dimensions = array<i64: 1>}} : ({T(M2)}) -> {T(R, M2)}
    %z9 = "stablehlo.add"(%y9, %c9) : ({T(R, M2)}, {T(R, M2)}) -> {T(R, M2)}
    func.return %z9 : {T(R, M2)}
  }}
}}
"""


def norm_text(R, C):
    """x [R, C] -> ggml.norm -> * gain -> + bias, the layer norm as the encoder writes it."""
    T = lambda *d: "tensor<" + "".join("%dx" % x for x in d) + "f32>"
    return f"""module {{
  func.func public @main(%x: {T(R, C)}, %g: {T(C)}, %be: {T(C)}) -> {T(R, C)} {{
    %n = "stablehlo.custom_call"(%x) {{call_target_name = "ggml.norm", backend_config = "eps = 0x{D.EPS_BITS:08X} : f32"}} : ({T(R, C)}) -> {T(R, C)}
    %gg = "stablehlo.broadcast_in_dim"(%g) {{broadcast_dimensions = array<i64: 1>}} : ({T(C)}) -> {T(R, C)}
    %t = "stablehlo.multiply"(%n, %gg) : ({T(R, C)}, {T(R, C)}) -> {T(R, C)}
    %bb = "stablehlo.broadcast_in_dim"(%be) {{broadcast_dimensions = array<i64: 1>}} : ({T(C)}) -> {T(R, C)}
    %a = "stablehlo.add"(%t, %bb) : ({T(R, C)}, {T(R, C)}) -> {T(R, C)}
    func.return %a : {T(R, C)}
  }}
}}
"""


@pytest.mark.parametrize("R,C,M2,linked", [
    (1100, 512, 1536, True),   # the packed norm (a partial last 32-row tile, padded rows); k_mul_mat_seg consumer
    (4000, 512, 1536, True),   # k_mul_mat_tm consumer
    (300, 1024, 512, True),    # eight float4 groups a lane
    (1100, 576, 512, True),    # a row not a multiple of 128: the block norm, then the pack kernel
    (1100, 1000, 512, False),  # K not a multiple of 64: no handoff
])
def test_norm_packed_handoff_matches_unfused(R, C, M2, linked, capfd, monkeypatch):
    """The layer norm (norm, gain, bias) writing its result in the next dense
    product's packed x layout, against the ops one at a time."""
    rng = np.random.default_rng(R + C + M2)
    args = [specials(rng, (R, C)), specials(rng, (C,)), specials(rng, (C,)),
            specials(rng, (M2, C)) * np.float32(0.05), specials(rng, (M2,))]
    args = [M.of_numpy(a) for a in args]
    T = lambda *d: "tensor<" + "".join("%dx" % x for x in d) + "f32>"
    l = E.load(then_dense(norm_text(R, C), R, C, M2, "%a", T(R, C)))
    want = M.to_numpy(E.call(E.prepare(l, None, False), args)[0])
    fn = E.prepare(l, None, True)
    got, chains, err = run_counted(capfd, monkeypatch, fn, args)
    assert chains == 2, err
    assert ("handing a packed operand on: 1" in err) == linked, err
    assert np.array_equal(bits(got), bits(want))
    assert np.array_equal(bits(M.to_numpy(E.call(fn, args)[0])), bits(want))


@pytest.mark.parametrize("B,S,H,M2", [
    (2, 256, 8, 512),    # the packed epilogue; k_mul_mat_seg consumer
    (8, 256, 8, 1536),   # k_mul_mat_tm consumer
    (3, 256, 2, 384),    # two heads: K = 128
    (1, 256, 1, 256),    # one head: the chain ends at the value product
    (2, 128, 4, 512),    # 128 positions: the pack kernel after the attention
])
def test_attention_packed_handoff_matches_unfused(B, S, H, M2, capfd, monkeypatch):
    """The fused attention writing the merged heads in the output projection's
    packed x layout, against the ops one at a time."""
    rng = np.random.default_rng(B * 7 + S + H + M2)
    K = H * 64
    args = [rng.standard_normal((B, S, 3, H, 64)).astype(np.float32), specials(rng, (M2, K)) * np.float32(0.05),
            specials(rng, (M2,))]
    args = [M.of_numpy(a) for a in args]
    T = lambda *d: "tensor<" + "".join("%dx" % x for x in d) + "f32>"
    l = E.load(then_dense(attn_text(B, S, H, 64, 0x3E000000, True), B * S, K, M2, "%r", T(B, S, K)))
    want = M.to_numpy(E.call(E.prepare(l, None, False), args)[0])
    fn = E.prepare(l, None, True)
    got, chains, err = run_counted(capfd, monkeypatch, fn, args)
    assert chains == 2, err
    assert "handing a packed operand on: 1" in err, err
    assert np.array_equal(bits(got), bits(want))
    assert np.array_equal(bits(M.to_numpy(E.call(fn, args)[0])), bits(want))
