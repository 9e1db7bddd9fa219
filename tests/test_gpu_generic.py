"""The generic path's region ops on the B200 (Lower.lean:317-470), compiled and
uncompiled, bit for bit against numpy:

* `while` unrolled at trace time (binary32, and binary64 on uint64 carriers
  through the soft-float kernels), and its planted fault (one iteration
  short) differing;
* `dynamic_slice` with starts known at trace time, clamped as StableHLO says;
* `gather` of a 1-D table with clamped indices;
* `reduce` with a maximum body over one axis or both;

and the refusals: a `while` condition or a `dynamic_slice` start that depends
on data, a `reduce` body other than a maximum, a gather of a 2-D table."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import generic_modules as GM  # noqa: E402
from shlo import exec as E  # noqa: E402
from shlo import lower as L  # noqa: E402
from shlo import mlx as M  # noqa: E402


def run(text, args, compile, faults=None):
    return [M.to_numpy(a) for a in E.call(E.prepare(E.load(text), faults, compile), args)]


def same(a, b):
    a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
    return a.shape == b.shape and np.array_equal(a.view(np.uint8), b.view(np.uint8))


@pytest.mark.parametrize("compile", [True, False])
@pytest.mark.parametrize("trips", [0, 1, 5])
def test_while_f32(trips, compile):
    rng = np.random.default_rng(trips)
    x = rng.standard_normal(300).astype(np.float32)
    y = (rng.standard_normal(300) * 1e-3).astype(np.float32)
    want = x.copy()
    for _ in range(trips):
        want = (want + y).astype(np.float32)
    got = run(GM.while_accumulate(300, trips), [M.of_numpy(x), M.of_numpy(y)], compile)[0]
    assert same(got, want)
    if trips:
        short = run(GM.while_accumulate(300, trips), [M.of_numpy(x), M.of_numpy(y)], compile,
                    L.Faults(whileShort=True))[0]
        assert not same(short, want)


@pytest.mark.parametrize("compile", [True, False])
def test_while_f64_soft_float(compile):
    rng = np.random.default_rng(7)
    x = rng.standard_normal(257) * 1e3
    y = rng.standard_normal(257) * np.pi
    want = x.copy()
    for _ in range(4):
        want = want + y
    got = run(GM.while_accumulate(257, 4, el="f64"), [M.of_numpy(x.view(np.uint64), M.dtU64),
                                                      M.of_numpy(y.view(np.uint64), M.dtU64)], compile)[0]
    assert same(got.view(np.float64), want)


@pytest.mark.parametrize("compile", [True, False])
@pytest.mark.parametrize("starts,size", [((2, 3, 1), (4, 4)), ((10, 9, 7), (5, 3)), ((0, 0, 0), (16, 8)),
                                         ((-4, 1, -2), (3, 2))])
def test_dynamic_slice_known_starts(starts, size, compile):
    rows, cols = 16, 8
    x = np.arange(rows * cols, dtype=np.float32).reshape(rows, cols) * np.float32(0.5)
    s0 = max(0, min(starts[0] + starts[1], rows - size[0]))
    s1 = max(0, min(starts[2], cols - size[1]))
    want = x[s0:s0 + size[0], s1:s1 + size[1]]
    got = run(GM.dynamic_slice(rows, cols, starts, size), [M.of_numpy(x)], compile)[0]
    assert same(got, want)


@pytest.mark.parametrize("compile", [True, False])
def test_gather1d_clamps(compile):
    rng = np.random.default_rng(3)
    table = rng.standard_normal(16).astype(np.float32)
    idx = np.array([0, 15, 3, -5, 16, 99, 7, 2, -1, 8], dtype=np.int64)
    got = run(GM.gather1d(16, idx.size), [M.of_numpy(table), M.of_numpy(idx)], compile)[0]
    assert same(got, table[np.clip(idx, 0, 15)])


@pytest.mark.parametrize("compile", [True, False])
@pytest.mark.parametrize("dims", [[1], [0], [0, 1]])
def test_reduce_max(dims, compile):
    rng = np.random.default_rng(len(dims) * 3 + dims[0])
    x = rng.standard_normal((37, 65)).astype(np.float32)
    x[5, 7] = -np.inf
    for init in (np.float32(-np.inf), np.float32(0.25)):
        want = np.maximum(np.max(x, axis=tuple(dims)), init).astype(np.float32)
        got = run(GM.reduce_max(37, 65, dims), [M.of_numpy(x), M.of_numpy(np.array(init, np.float32))], compile)[0]
        assert same(got, want)


def refused(text, args, needle):
    with pytest.raises(M.ShloError) as e:
        run(text, args, True)
    assert needle in str(e.value), str(e.value)


def test_refusals():
    x = M.of_numpy(np.ones(8, np.float32))
    refused(GM.while_accumulate(8, 3, cond_from_data=True), [x, x, M.of_numpy(np.array(3, np.int64))],
            "depends on data")
    refused(GM.dynamic_slice(16, 8, (1, 1, 0), (2, 2), from_data=True),
            [M.of_numpy(np.ones((16, 8), np.float32)), M.of_numpy(np.array(1, np.int64))], "depends on data")
    refused(GM.reduce_max(4, 8, [1], body="stablehlo.add"),
            [M.of_numpy(np.ones((4, 8), np.float32)), M.of_numpy(np.array(0, np.float32))], "maximum")
    refused(GM.gather1d(16, 4, table_rank2=True),
            [M.of_numpy(np.ones((16, 1), np.float32)), M.of_numpy(np.zeros(4, np.int64))], "1-D table")
