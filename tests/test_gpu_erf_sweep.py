"""The exhaustive erff check of Tests/OpTests.lean:273-296:
all 2^32 binary32 inputs, NaN, infinities and subnormals included.

Chunk by chunk (2^24 inputs), the GPU kernel erff_map is compared on the
device with the oracle's correctly rounded erff computed on the host cores
(erfl, with binary128 re-evaluation near rounding midpoints: a method
independent of the kernel's binary64 Taylor expansion): `binary ne` then
`count_nonzero`, as the reference does. Then the planted fault: the CPU side
shifted by one input must differ.
"""
import concurrent.futures as cf
import os
import time

import numpy as np
import pytest

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

from oracle import oracle as O  # noqa: E402
from shlo import mlx as M  # noqa: E402
from shlo import run as Run  # noqa: E402

CHUNK_LOG = 24


def test_erff_exhaustive():
    chunk = 1 << CHUNK_LOG
    chunks = (1 << 32) // chunk
    workers = max(1, os.cpu_count() or 1)
    bad, first_bad = 0, None
    t0 = time.perf_counter()
    gpu_s = 0.0
    with cf.ThreadPoolExecutor(max_workers=workers) as ex:
        futs = {ex.submit(O.erff_range, c * chunk, chunk, 1): c for c in range(chunks)}
        for fut in cf.as_completed(futs):
            c = futs[fut]
            base = c * chunk
            g0 = time.perf_counter()
            gpu = Run.erff_map(base, chunk)
            M.eval_([gpu])
            gpu_s += time.perf_counter() - g0
            cpu = M.of_numpy(fut.result(), M.dtU32)
            k = M.count_nonzero(M.binary(M.opNe, gpu, cpu))
            if k:
                bad += k
                first_bad = base if first_bad is None else min(first_bad, base)
    dt = time.perf_counter() - t0
    print("erff_exhaustive: %d of 4294967296 differ (%.1f s; GPU erff_map %.2f s, %.3g patterns/s)"
          % (bad, dt, gpu_s, 2.0 ** 32 / gpu_s))
    assert bad == 0, "first differing chunk at %08x" % first_bad
    # Planted: compare against the CPU routine one input late.
    gpu = Run.erff_map(0x3F000000, chunk)
    cpu = M.of_numpy(O.erff_range(0x3F000001, chunk), M.dtU32)
    assert M.count_nonzero(M.binary(M.opNe, gpu, cpu)) != 0
