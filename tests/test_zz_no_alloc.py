"""shlo_mul_mat_noalloc: mul_mat for callers that cannot let this library
allocate device memory (their GPU memory belongs to their own pool or arena).

The entry point is called through the C ABI with caller-owned device buffers,
twice in a row on each shape (the calls share one scratch array, so the second
must not see the first's leftovers), and its output must equal the allocating
"smlx_mul_mat" kernel's word for word -- the zero tolerance of every mul_mat
test here. A shape whose packed operands exceed the scratch maximum must be
refused with an error. This file is collected last on purpose."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

from shlo import _lib  # noqa: E402
from shlo import mlx as M  # noqa: E402
from shlo import run as Run  # noqa: E402

SHAPES = [  # K, M, R, N, batched
    (512, 256, 300, 300, False),   # packed fast path, K a multiple of 16
    (737, 96, 64, 64, False),      # with a tail
    (64, 256, 512, 256, True),     # batched w, as attention uses it
    (7, 33, 20, 20, False),        # K < 16: all tail, no scratch needed
]


def call_noalloc(w, x, K, Mm, R, N, wbs):
    L = _lib.load()
    dev = torch.device("cuda", 0)
    wt = torch.from_numpy(w).to(dev)
    xt = torch.from_numpy(x).to(dev)
    yt = torch.empty(R * Mm, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    rc = L.shlo_mul_mat_noalloc(wt.data_ptr(), xt.data_ptr(), yt.data_ptr(), K, Mm, R, N, wbs,
                                ctypes.c_void_p(stream.cuda_stream))
    _lib.check(rc)
    stream.synchronize()
    return yt.cpu().numpy()


@pytest.mark.parametrize("K,Mm,R,N,batched", SHAPES)
def test_noalloc_matches_allocating_kernel_twice(K, Mm, R, N, batched):
    M.set_device(0)
    M.set_flavor("pinned")
    rng = np.random.default_rng(K + Mm + R)
    wb = R // N if batched else 1
    wbs = Mm * K if batched else 0
    for call in range(2):
        w = rng.standard_normal((wb, Mm, K)).astype(np.float32)
        x = rng.standard_normal((R, K)).astype(np.float32)
        want = M.to_numpy(Run.mul_mat(M.of_numpy(w), M.of_numpy(x), K, Mm, R, N, wbs))
        got = call_noalloc(w, x, K, Mm, R, N, wbs)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), "call %d differs" % call


def test_noalloc_refuses_shapes_beyond_its_scratch():
    K, Mm, R = 2048, 1024, 2048  # packed operands: 16 MiB + 8 MiB
    w = np.zeros((Mm, K), np.float32)
    x = np.zeros((R, K), np.float32)
    with pytest.raises(_lib.ShloError, match="scratch"):
        call_noalloc(w, x, K, Mm, R, R, 0)
