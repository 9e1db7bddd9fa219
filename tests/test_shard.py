"""Multi-GPU host logic on the CPU: the partition rules and the host-side
collectives (sum, max, the final gather) over two gloo ranks."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from shlo import shard as S


@pytest.mark.parametrize("n", [0, 1, 7, 64, 1000, 1 << 32])
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_split_partitions(n, world):
    spans = [S.split(n, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    for (a, b), (c, d) in zip(spans, spans[1:]):
        assert b == c and a <= b
    sizes = [b - a for a, b in spans]
    assert max(sizes) - min(sizes) <= 1


def test_round_robin_and_sweep_chunks():
    items = list(range(38))
    parts = [S.round_robin(items, 4, r) for r in range(4)]
    assert sorted(sum(parts, [])) == items
    lo, hi = S.sweep_range(8, 7)
    assert hi == 1 << 32 and lo == 7 << 29
    ch = S.sweep_chunks(lo, hi)
    assert ch[0][0] == lo and sum(c for _, c in ch) == hi - lo and max(c for _, c in ch) == 1 << 24
    with pytest.raises(ValueError):
        S.split(10, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        # the denoiser batch: rows [lo, hi) of a 10-sample global batch, gathered at rank 0
        lo, hi = S.split(10, world, rank)
        local = np.arange(lo * 3, hi * 3, dtype=np.float32).reshape(hi - lo, 3)
        got = S.gather_rows(dist, local, world, rank)
        # the sweep: a mismatch count per rank, summed (here: patterns whose low byte is 0x5A in a sample)
        slo, shi = S.sweep_range(world, rank)
        sample = np.arange(slo, shi, 1 << 16, dtype=np.uint64)
        count = int(np.count_nonzero((sample >> np.uint64(16)) & np.uint64(0xFF) == 0x5A))
        total = S.sum_over_ranks(dist, count)
        slowest = S.max_over_ranks(dist, 1.5 + rank)
        q.put((rank, None if got is None else got.tolist(), total, slowest))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r = q.get(timeout=120)
        res[r[0]] = r
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0][1] == np.arange(30, dtype=np.float32).reshape(10, 3).tolist()
    assert res[1][1] is None
    sample = np.arange(0, 1 << 32, 1 << 16, dtype=np.uint64)
    want = int(np.count_nonzero((sample >> np.uint64(16)) & np.uint64(0xFF) == 0x5A))
    assert res[0][2] == res[1][2] == want
    assert res[0][3] == res[1][3] == 2.5


def _leaving_worker(rank, world, port, q):
    """Rank 1 leaves before the job's collective (a host-side failure: the
    process returns between steps, nothing of it in flight); rank 0's collective
    must end with an error within its short timeout instead of waiting for good."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    import time
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        q.put((1, "left"))
        q.close()
        q.join_thread()  # the message is out before the process goes
        os._exit(0)  # gone without the collective or the group's teardown
    t0 = time.monotonic()
    try:
        S.sum_over_ranks(dist, 3)
        q.put((0, "no error", time.monotonic() - t0))
    except Exception as e:  # the collective's timeout or the peer's closed connection
        q.put((0, type(e).__name__, time.monotonic() - t0))


def test_a_rank_that_leaves_is_detected_not_waited_for():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaving_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r = q.get(timeout=120)
        res[r[0]] = r
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res[1][1] == "left"
    assert res[0][1] != "no error", res[0]
    assert res[0][2] < 60, res[0]  # ended by the group's 5 s limit (or at once), not the test's
