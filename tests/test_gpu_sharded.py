"""The sharded harness (tests/multi_gpu.py) on every GPU this box gives: the
exhaustive erf sweep split into contiguous ranges and the 38 ggml cases dealt
round robin, one process per GPU, results summed / gathered to rank 0. On a
one-GPU box this is the N = 1 case of the same code."""
import json
import os
import socket
import subprocess
import sys

import pytest

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

HERE = os.path.dirname(os.path.abspath(__file__))


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_sharded_sweep_and_cases():
    import torch
    n = max(1, min(8, torch.cuda.device_count()))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes", "1", "--nproc-per-node", str(n),
           "--master-addr", "127.0.0.1", "--master-port", str(free_port()),
           os.path.join(HERE, "multi_gpu.py"), "--what", "sweep,cases"]
    r = subprocess.run(["timeout", "-k", "30", "900"] + cmd, capture_output=True, text=True)
    lines = [json.loads(x) for x in r.stdout.splitlines() if x.startswith("{")]
    assert r.returncode == 0, (r.stdout[-2000:], r.stderr[-3000:])
    by = {x["what"]: x for x in lines}
    assert by["erf-sweep"]["mismatches"] == 0 and by["erf-sweep"]["planted_fault_caught_on_ranks"] == n
    assert by["op-cases"]["cases"] == 38 and by["op-cases"]["passed"] == 38, by["op-cases"]["failed"]
    print(json.dumps(lines))
