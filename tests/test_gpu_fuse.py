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
