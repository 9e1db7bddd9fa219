"""Compiled functions (Mlx.lean:66-67, `compile` with enable = 1): the first call
of each input signature is recorded as a CUDA graph, later calls replay it.

The reference's contract for a compiled function is MLX's: the same results as
calling the function, for any inputs of the recorded shapes, and every result
an independent immutable array. These tests hold the replay path to that, bit
for bit, against eager calls of the same function.
"""
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
    return np.ascontiguousarray(a).view(np.uint32)


@pytest.fixture(autouse=True)
def _pinned():
    M.set_flavor("pinned")
    yield


def mm_fn(args):
    w, x = args
    y = Run.mul_mat(w, x, 64, 48, 300, 300, 0)
    return [M.binary(M.opAdd, y, y), Run.soft_max(M.reshape(y, [300, 48]), 48, 300, 0x3F800000)]


def test_replay_matches_eager_for_new_inputs():
    rng = np.random.default_rng(1)
    w = M.of_numpy(rng.standard_normal((48, 64)).astype(np.float32))
    fg = M.compile_(mm_fn, True)
    fe = M.compile_(mm_fn, False)
    for step in range(4):
        x = M.of_numpy(rng.standard_normal((300, 64)).astype(np.float32))
        got = [M.to_numpy(a) for a in M.apply(fg, [w, x])]
        want = [M.to_numpy(a) for a in M.apply(fe, [w, x])]
        for g, e in zip(got, want):
            assert np.array_equal(bits(g), bits(e)), "step %d" % step


def test_results_stay_independent():
    rng = np.random.default_rng(2)
    w = M.of_numpy(rng.standard_normal((48, 64)).astype(np.float32))
    fg = M.compile_(mm_fn, True)
    x1 = M.of_numpy(rng.standard_normal((300, 64)).astype(np.float32))
    x2 = M.of_numpy(rng.standard_normal((300, 64)).astype(np.float32))
    o1 = M.apply(fg, [w, x1])
    first = M.to_numpy(o1[0]).copy()
    o2 = M.apply(fg, [w, x2])
    M.eval_(o2)
    assert np.array_equal(bits(M.to_numpy(o1[0])), bits(first))
    assert not np.array_equal(M.to_numpy(o2[0]), first)


def test_new_weights_rederive_the_packed_layout():
    """The packed weight cached on the private input copy is derived again when
    a replay brings a different weight array."""
    rng = np.random.default_rng(3)
    x = M.of_numpy(rng.standard_normal((300, 64)).astype(np.float32))
    fg = M.compile_(mm_fn, True)
    fe = M.compile_(mm_fn, False)
    for _ in range(3):
        w = M.of_numpy(rng.standard_normal((48, 64)).astype(np.float32))
        got = M.to_numpy(M.apply(fg, [w, x])[0])
        want = M.to_numpy(M.apply(fe, [w, x])[0])
        assert np.array_equal(bits(got), bits(want))


def test_strided_inputs_and_new_signatures():
    def f(args):
        return [M.binary(M.opMul, args[0], args[0])]
    fg = M.compile_(f, True)
    a = np.arange(24, dtype=np.float32).reshape(4, 6)
    t = M.transpose(M.of_numpy(a), [1, 0])  # a strided view
    assert np.array_equal(M.to_numpy(M.apply(fg, [t])[0]), (a * a).T)
    b = np.arange(10, dtype=np.float32)
    assert np.array_equal(M.to_numpy(M.apply(fg, [M.of_numpy(b)])[0]), b * b)  # a second signature
    assert np.array_equal(M.to_numpy(M.apply(fg, [t])[0]), (a * a).T)


def test_identity_output_and_constants():
    def f(args):
        c = M.of_numpy(np.full((5,), 3.0, np.float32))  # a constant made while recording
        return [args[0], M.binary(M.opAdd, args[0], c)]
    fg = M.compile_(f, True)
    for v in (1.0, 2.0, 7.0):
        x = np.full((5,), v, np.float32)
        o = M.apply(fg, [M.of_numpy(x)])
        assert np.array_equal(M.to_numpy(o[0]), x)
        assert np.array_equal(M.to_numpy(o[1]), x + 3.0)


def test_a_function_that_waits_runs_eagerly():
    """eval inside the function cannot be recorded: that signature falls back to
    calling the function, with the same results."""
    def f(args):
        y = M.binary(M.opAdd, args[0], args[0])
        M.eval_([y])
        return [y]
    fg = M.compile_(f, True)
    for v in (1.0, 4.0):
        x = np.full((8,), v, np.float32)
        assert np.array_equal(M.to_numpy(M.apply(fg, [M.of_numpy(x)])[0]), 2 * x)


def test_replay_counts_the_recorded_launches():
    rng = np.random.default_rng(4)
    w = M.of_numpy(rng.standard_normal((48, 64)).astype(np.float32))
    x = M.of_numpy(rng.standard_normal((300, 64)).astype(np.float32))
    fe = M.compile_(mm_fn, False)
    M.eval_(M.apply(fe, [w, x]))  # packs and caches w
    c0 = M.launch_count()
    M.eval_(M.apply(fe, [w, x]))
    eager = M.launch_count() - c0
    fg = M.compile_(mm_fn, True)
    M.eval_(M.apply(fg, [w, x]))  # records
    c1 = M.launch_count()
    M.eval_(M.apply(fg, [w, x]))  # replays: the graph, plus one copy per result
    assert M.launch_count() - c1 == eager + 2


def test_denoiser_module_compiled_equals_eager():
    cfg = D.Config(layers=2)
    B = 2
    w = D.init_weights(cfg, seed=5)
    W = [M.of_numpy(w[n]) for n, _ in D.weight_specs(cfg)]
    text = D.module_text(cfg, B)
    fg = E.prepare(E.load(text), None, True)
    fe = E.prepare(E.load(text), None, False)
    for seed in (1, 2, 3):
        X = [M.of_numpy(a) for a in D.inputs(cfg, B, seed=seed)]
        got = M.to_numpy(E.call(fg, X + W)[0])
        want = M.to_numpy(E.call(fe, X + W)[0])
        assert np.array_equal(bits(got), bits(want)), "seed %d" % seed
