"""Reshape of strided views (slices, transposes, broadcasts): a view when the
strides allow it, a copy otherwise; the values are numpy's either way."""
import numpy as np
import pytest

from shlo import mlx as M

pytestmark = pytest.mark.gpu

CASES = [
    # (base shape, view builder (numpy and shlo), new shape)
    ((2, 5, 3, 4, 6), lambda a, m: (a[:, :, 1:2], m.slice_(a_m(m), [0, 0, 1, 0, 0], [2, 5, 2, 4, 6], [1] * 5)), (2, 5, 4, 6)),
    ((2, 5, 3, 4, 6), lambda a, m: (a[:, :, 1:2], m.slice_(a_m(m), [0, 0, 1, 0, 0], [2, 5, 2, 4, 6], [1] * 5)), (10, 24)),
    ((2, 5, 3, 4, 6), lambda a, m: (a[:, :, 2:3], m.slice_(a_m(m), [0, 0, 2, 0, 0], [2, 5, 3, 4, 6], [1] * 5)), (2, 5, 24)),
    ((4, 6, 8), lambda a, m: (a.transpose(1, 0, 2), m.transpose(a_m(m), [1, 0, 2])), (6, 32)),
    ((4, 6, 8), lambda a, m: (a.transpose(1, 0, 2), m.transpose(a_m(m), [1, 0, 2])), (24, 8)),
    ((4, 6, 8), lambda a, m: (a.transpose(2, 1, 0), m.transpose(a_m(m), [2, 1, 0])), (8, 24)),
    ((6, 8), lambda a, m: (a[:, 2:6], m.slice_(a_m(m), [0, 2], [6, 6], [1, 1])), (6, 2, 2)),
    ((6, 8), lambda a, m: (a[:, 2:6], m.slice_(a_m(m), [0, 2], [6, 6], [1, 1])), (24,)),
    ((6, 8), lambda a, m: (a[::2, :], m.slice_(a_m(m), [0, 0], [6, 8], [2, 1])), (3, 2, 4, 1)),
    ((1, 8), lambda a, m: (np.broadcast_to(a, (5, 8)), m.broadcast(a_m(m), [5, 8])), (40,)),
]

_state = {}


def a_m(m):
    return _state["arr"]


@pytest.mark.parametrize("i", range(len(CASES)))
def test_reshape_of_views(i):
    shape, build, new = CASES[i]
    a = np.arange(int(np.prod(shape)), dtype=np.float32).reshape(shape) * 0.5
    _state["arr"] = M.of_numpy(a)
    npv, mv = build(a, M)
    got = M.to_numpy(M.reshape(mv, list(new)))
    assert np.array_equal(got, np.reshape(npv, new))
    # and the reshaped view feeds an op correctly
    got2 = M.to_numpy(M.binary(M.opAdd, M.reshape(mv, list(new)), M.reshape(mv, list(new))))
    assert np.array_equal(got2, 2 * np.reshape(npv, new))
