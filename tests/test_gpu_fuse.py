"""The executor's fused launches (shlo/fuse.py) against the unfused sequence
they replace, bit for bit: the fused kernels alone on random data with
specials, and whole modules (the encoder layer and the denoiser) fused and
unfused."""
from __future__ import annotations

import numpy as np
import pytest

import shlo  # noqa: F401
from shlo import denoiser as D
from shlo import exec as E
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


@pytest.mark.parametrize("cfg,B", [(D.ENCODER, 2), (D.Config(layers=2), 3)])
def test_modules_fused_equal_unfused(cfg, B):
    w = D.init_weights(cfg, seed=9)
    W = [M.of_numpy(w[n]) for n, _ in D.weight_specs(cfg)]
    X = [M.of_numpy(a) for a in D.inputs(cfg, B, seed=4)]
    text = D.module_text(cfg, B)
    fused = E.load(text)
    plain = E.load(text)
    plain.module.fuse = False
    for compile_ in (False, True):
        got = M.to_numpy(E.call(E.prepare(fused, None, compile_), X + W)[0])
        want = M.to_numpy(E.call(E.prepare(plain, None, compile_), X + W)[0])
        assert np.array_equal(bits(got), bits(want))


def attn_text(B, S, H, W, scale_bits):
    T = lambda *d: "tensor<" + "".join("%dx" % x for x in d) + "f32>"
    q, s_, o, qkv = T(B, S, H, W), T(B, H, S, S), T(B, H, S, W), T(B, S, 3, H, W)
    sl = T(B, S, 1, H, W)
    parts = []
    for i in range(3):
        parts.append(
            f'    %sl{i} = "stablehlo.slice"(%qkv) {{start_indices = array<i64: 0, 0, {i}, 0, 0>, limit_indices = '
            f'array<i64: {B}, {S}, {i + 1}, {H}, {W}>, strides = array<i64: 1, 1, 1, 1, 1>}} : ({qkv}) -> {sl}\n'
            f'    %x{i} = "stablehlo.reshape"(%sl{i}) : ({sl}) -> {q}\n')
    return f"""module {{
  func.func public @main(%qkv: {qkv}) -> ({q}) {{
{''.join(parts)}    %s = "stablehlo.dot_general"(%x0, %x1) {{dot_dimension_numbers = #stablehlo.dot<lhs_batching_dimensions = [0, 2], rhs_batching_dimensions = [0, 2], lhs_contracting_dimensions = [3], rhs_contracting_dimensions = [3]>}} : ({q}, {q}) -> {s_}
    %p = "stablehlo.custom_call"(%s) {{call_target_name = "ggml.soft_max", backend_config = "scale = 0x{scale_bits:08X} : f32"}} : ({s_}) -> {s_}
    %o = "stablehlo.dot_general"(%p, %x2) {{dot_dimension_numbers = #stablehlo.dot<lhs_batching_dimensions = [0, 1], rhs_batching_dimensions = [0, 2], lhs_contracting_dimensions = [3], rhs_contracting_dimensions = [1]>}} : ({s_}, {q}) -> {o}
    %t = "stablehlo.transpose"(%o) {{permutation = array<i64: 0, 2, 1, 3>}} : ({o}) -> {q}
    func.return %t : {q}
  }}
}}
"""


@pytest.mark.parametrize("B,S,H,scale,special,amp", [(2, 256, 8, 0x3E000000, False, 4.0), (1, 128, 3, 0x3E000000, True, 4.0),
                                                     (3, 256, 2, 0x3F800000, True, 4.0), (1, 256, 1, 0x41000000, False, 4.0),
                                                     (2, 256, 4, 0x3E000000, False, 0.05), (1, 128, 2, 0x3E000000, False, 0.3),
                                                     (2, 256, 2, 0x3E000000, False, 1.0)])
def test_attention_matches_unfused(B, S, H, scale, special, amp):
    # q, k, v as the strided slices of one projection, as in the encoder layer;
    # specials give NaN and infinite score rows (the soft_max's sequential scan);
    # small amplitudes keep every row's exponentials within a few binades (the
    # group sums added in any order), large ones spread them (the serial chain)
    rng = np.random.default_rng(B * 1000 + S + H)
    a = specials(rng, (B, S, 3, H, 64)) if special else rng.standard_normal((B, S, 3, H, 64)).astype(np.float32)
    x = [M.of_numpy(a * np.float32(amp))]
    text = attn_text(B, S, H, 64, scale)
    fused = E.load(text)
    plain = E.load(text)
    plain.module.fuse = False
    for compile_ in (False, True):
        got = M.to_numpy(E.call(E.prepare(fused, None, compile_), x)[0])
        want = M.to_numpy(E.call(E.prepare(plain, None, compile_), x)[0])
        assert np.array_equal(bits(got), bits(want))
