"""Failure detection without a GPU fault: the library's wait for the device
(`shlo_eval`, Mlx.lean's `eval`) is bounded by SHLO_EVAL_TIMEOUT_S and reports
an error when the work it waits for has not finished in time, instead of
waiting for good; the context stays usable, and once the work has finished the
same arrays read back correctly. The slow work is ordinary queued kernels (a
long run of exact mul_mat launches), never a hung or faulting one. Run in a
child process, since the limit is read once per process."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r'''
import sys, time
sys.path[:0] = [%r, %r]
import numpy as np
from shlo import mlx as M, run as Run
M.set_device(0)
rng = np.random.default_rng(0)
w = M.of_numpy(rng.standard_normal((2048, 2048)).astype(np.float32))
x = M.of_numpy(rng.standard_normal((16384, 2048)).astype(np.float32))
ys = [Run.mul_mat(w, x, 2048, 2048, 16384, 16384, 0) for _ in range(12)]  # ~40 ms of queued work
try:
    M.eval_(ys)
    print("RESULT no-timeout")
except M.ShloError as e:
    print("RESULT timeout", "did not finish within" in str(e))
time.sleep(2.0)  # the queued work ends on its own
M.eval_(ys)
a = M.to_numpy(M.slice_(ys[0], [0], [4096], [1])).view(np.uint32)  # small reads: quick under the limit
b = M.to_numpy(M.slice_(ys[-1], [0], [4096], [1])).view(np.uint32)
small = M.to_numpy(Run.mul_mat(M.of_numpy(np.ones((64, 32), np.float32)), M.of_numpy(np.ones((16, 32), np.float32)),
                               32, 64, 16, 16, 0))
print("RESULT after", bool(np.array_equal(a, b)), float(small[0]))
''' % (ROOT, os.path.join(ROOT, "contract-stablehlo-mlx_b200"))


def test_eval_limit_reports_an_error_and_the_context_survives():
    env = dict(os.environ, SHLO_EVAL_TIMEOUT_S="0.005")
    r = subprocess.run([sys.executable, "-c", CHILD], capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, r.stdout + r.stderr
    lines = [ln.split()[1:] for ln in r.stdout.splitlines() if ln.startswith("RESULT")]
    assert lines[0] == ["timeout", "True"], r.stdout
    assert lines[1] == ["after", "True", "32.0"], r.stdout
