"""Host transfers beside compute: pinned inputs of ofBytes (above 256 bytes) are uploaded on
the library's copy stream into blocks of their own pool, and toBytes reads a
compiled function's result on the copy stream after that result's ready event,
so both run while other work is queued on the compute stream. These tests
check that no upload lands in a block that queued compute still reads, and that
a result read back while the next call computes is that result, bit for bit."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import shlo  # noqa: F401
from shlo import mlx as M
from shlo import run as Run

pytestmark = pytest.mark.gpu


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


@pytest.fixture(autouse=True)
def _pinned():
    M.set_flavor("pinned")
    yield


def upload(t: torch.Tensor):
    return M.of_ptr(t.data_ptr(), t.numel() * 4, list(t.shape), M.dtF32)


def test_uploads_reuse_blocks_safely():
    # each round uploads new data while the previous rounds' products are still
    # queued, and drops its input at once: the upload pool must not hand a block
    # to the copy stream before the compute that reads it has run
    rng = np.random.default_rng(3)
    K, Mm, R = 512, 512, 2048  # x: 4 MiB, above the upload threshold
    w = M.of_numpy((rng.standard_normal((Mm, K)) * 0.05).astype(np.float32))
    host = [torch.from_numpy(rng.standard_normal((R, K)).astype(np.float32)).pin_memory() for _ in range(3)]
    outs, wants = [], []
    for i in range(12):
        src = host[i % 3]
        src.copy_(torch.from_numpy(rng.standard_normal((R, K)).astype(np.float32)))
        x = upload(src)
        outs.append(Run.mul_mat(w, x, K, Mm, R, R, 0))
        wants.append(src.numpy().copy())
        del x
    for o, xh in zip(outs, wants):
        want = M.to_numpy(Run.mul_mat(w, M.of_numpy(xh), K, Mm, R, R, 0))
        assert np.array_equal(bits(M.to_numpy(o)), bits(want))


def test_pipelined_readback_of_compiled_results():
    # the bench's end-to-end loop: step i's result read once step i + 1 is queued
    rng = np.random.default_rng(4)
    K, Mm, R = 256, 256, 4096

    def step(args):
        w, x = args
        y = Run.mul_mat(w, x, K, Mm, R, R, 0)
        return [Run.soft_max(M.reshape(y, [R, Mm]), Mm, R, 0x3F800000)]

    fn = M.compile_(step, True)
    w = M.of_numpy((rng.standard_normal((Mm, K)) * 0.05).astype(np.float32))
    xs = [rng.standard_normal((R, K)).astype(np.float32) for _ in range(4)]
    pin = torch.from_numpy(xs[0]).pin_memory()
    out = torch.empty((R, Mm), dtype=torch.float32).pin_memory()
    got, prev = [], None
    for x in xs:
        pin.copy_(torch.from_numpy(x))
        o = M.apply(fn, [w, upload(pin)])[0]
        if prev is not None:
            M.to_ptr(prev, out.data_ptr(), out.numel() * 4)
            got.append(out.numpy().copy())
        prev = o
    M.to_ptr(prev, out.data_ptr(), out.numel() * 4)
    got.append(out.numpy().copy())
    for g, x in zip(got, xs):
        want = M.to_numpy(step([w, M.of_numpy(x)])[0]).reshape(R, Mm)
        assert np.array_equal(bits(g), bits(want))


def test_small_uploads_beside_queued_compute():
    # small pinned inputs (a timestep embedding's size) take the upload path too:
    # each is added to a product still queued on the compute stream
    rng = np.random.default_rng(5)
    K, Mm, R = 512, 512, 4096
    w = M.of_numpy((rng.standard_normal((Mm, K)) * 0.05).astype(np.float32))
    x = M.of_numpy(rng.standard_normal((R, K)).astype(np.float32))
    small = torch.empty(Mm, dtype=torch.float32).pin_memory()
    outs, wants = [], []
    for i in range(8):
        y = Run.mul_mat(w, x, K, Mm, R, R, 0)  # queued
        v = rng.standard_normal(Mm).astype(np.float32)
        small.copy_(torch.from_numpy(v))
        b = upload(small)
        outs.append(M.binary(M.opAdd, M.reshape(y, [R, Mm]), M.broadcast(M.reshape(b, [1, Mm]), [R, Mm])))
        wants.append(v)
        del b
    y = M.to_numpy(Run.mul_mat(w, x, K, Mm, R, R, 0)).reshape(R, Mm)
    for o, v in zip(outs, wants):
        want = (y + v[None, :]).astype(np.float32)
        assert np.array_equal(bits(M.to_numpy(o)), bits(want))
