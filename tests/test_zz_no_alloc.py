"""shlo_mul_mat_noalloc: mul_mat for callers that cannot let this library
allocate device memory (their GPU memory belongs to their own pool or arena,
or they must not allocate while they record work).

The entry point is called through the C ABI with caller-owned device buffers.
Its output must equal the oracle's and the allocating "smlx_mul_mat" kernel's
word for word -- the zero tolerance of every mul_mat test here -- on shapes
that differ in K, in the packed segment length, in the padding of M and R, with
and without a tail and a batched w, in both ggml builds. The shapes run one
after another and then again in reverse order, so every call follows one whose
leftovers in the shared scratch array differ from its own. Free device memory
must not change across calls (nothing is allocated), and a shape whose packed
operands exceed the scratch maximum must be refused with an error. This file
is collected last on purpose."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from oracle import oracle as O  # noqa: E402
from shlo import _lib  # noqa: E402
from shlo import mlx as M  # noqa: E402
from shlo import run as Run  # noqa: E402

SHAPES = [  # K, M, R, N, batched
    (1000, 1000, 1000, 1000, False),  # the largest here: 8 MiB of packed operands
    (737, 96, 64, 64, False),         # a tail of 1, M and R padded
    (100, 200, 90, 30, True),         # batched w with a tail of 4, M not a multiple of 128
    (512, 256, 300, 300, False),      # K a multiple of 16
    (64, 256, 512, 256, True),        # batched w, as attention uses it
    (7, 33, 20, 20, False),           # K < 16: all tail, no scratch needed
    (2048, 130, 200, 200, False),     # long K, M just above a tile
]


class Case:
    """Seeded operands of one shape as caller-owned device buffers."""

    def __init__(self, K, Mm, R, N, batched):
        self.K, self.Mm, self.R, self.N = K, Mm, R, N
        self.wbs = Mm * K if batched else 0
        rng = np.random.default_rng(K * 31 + Mm * 7 + R)
        self.w = rng.standard_normal((R // N if batched else 1, Mm, K)).astype(np.float32)
        self.x = rng.standard_normal((R, K)).astype(np.float32)
        dev = torch.device("cuda", 0)
        self.wt = torch.from_numpy(self.w).to(dev)
        self.xt = torch.from_numpy(self.x).to(dev)
        self.yt = torch.empty(R * Mm, dtype=torch.float32, device=dev)

    def call(self):
        stream = torch.cuda.current_stream(self.yt.device)
        self.yt.fill_(float("nan"))
        rc = _lib.load().shlo_mul_mat_noalloc(self.wt.data_ptr(), self.xt.data_ptr(), self.yt.data_ptr(), self.K,
                                              self.Mm, self.R, self.N, self.wbs, ctypes.c_void_p(stream.cuda_stream))
        _lib.check(rc)
        stream.synchronize()
        return self.yt.cpu().numpy()

    def want(self, flavor):
        oracle = O.mul_mat(self.w, self.x, self.K, self.Mm, self.R, self.N, self.wbs,
                           O.PINNED if flavor == "pinned" else O.STOCK)
        alloc = M.to_numpy(Run.mul_mat(M.of_numpy(self.w), M.of_numpy(self.x), self.K, self.Mm, self.R, self.N,
                                       self.wbs))
        return oracle, alloc


def same(a, b):
    return np.array_equal(np.ascontiguousarray(a).view(np.uint32).reshape(-1),
                          np.ascontiguousarray(b).view(np.uint32).reshape(-1))


@pytest.fixture(scope="module")
def cases():
    torch.cuda.set_device(0)
    M.set_device(0)
    return [Case(*s) for s in SHAPES]


@pytest.mark.parametrize("flavor", ["pinned", "stock"])
def test_noalloc_matches_oracle_and_allocating_kernel(cases, flavor):
    M.set_flavor(flavor)
    try:
        wants = [c.want(flavor) for c in cases]
        order = list(range(len(cases))) + list(reversed(range(len(cases))))
        for i in order:
            got = cases[i].call()
            oracle, alloc = wants[i]
            assert same(oracle, alloc), "the allocating kernel differs from the oracle on %s" % (SHAPES[i],)
            assert same(got, oracle), "noalloc differs on %s (%s build)" % (SHAPES[i], flavor)
    finally:
        M.set_flavor("pinned")


def test_noalloc_allocates_nothing(cases):
    M.set_flavor("pinned")
    for c in cases:  # the first calls load the kernels and look up the scratch address
        c.call()
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info(0)[0]
    for _ in range(3):
        for c in cases:
            c.call()
    torch.cuda.synchronize()
    free1 = torch.cuda.mem_get_info(0)[0]
    assert free1 == free0, "free device memory changed by %d bytes" % (free0 - free1)


def test_noalloc_refuses_shapes_beyond_its_scratch():
    M.set_device(0)
    K, Mm, R = 2048, 1024, 2048  # packed operands: 16 MiB + 8 MiB
    dev = torch.device("cuda", 0)
    w = torch.zeros(Mm * K, device=dev)
    x = torch.zeros(R * K, device=dev)
    y = torch.zeros(R * Mm, device=dev)
    rc = _lib.load().shlo_mul_mat_noalloc(w.data_ptr(), x.data_ptr(), y.data_ptr(), K, Mm, R, R, 0, None)
    assert rc != 0
    assert "scratch" in _lib.load().shlo_last_error().decode()
