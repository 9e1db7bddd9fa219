"""Partitioning the hot path's independent work over the GPUs of one node.

Nothing on the path exchanges data between units (a denoiser sample, a ggml
op case, a range of erf bit patterns), so each rank (one process per GPU)
takes a disjoint share and runs it alone; the only collectives are on the
host side: a sum of counts, a max of times, and one final gather of results
to rank 0. The process group is whatever the caller initialised (gloo for the
host control plane; the same calls work over NCCL).
"""
from __future__ import annotations

from typing import List, Sequence, Tuple

import numpy as np

SWEEP_PATTERNS = 1 << 32


def split(n: int, world: int, rank: int) -> Tuple[int, int]:
    """Rank `rank`'s contiguous share [lo, hi) of n units; the first n % world
    ranks take one extra unit."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank %d of %d" % (rank, world))
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def round_robin(items: Sequence, world: int, rank: int) -> list:
    """Every world-th item starting at `rank` (the op cases: shapes differ, so
    interleaving balances the work better than contiguous blocks)."""
    return [x for i, x in enumerate(items) if i % world == rank]


def sweep_range(world: int, rank: int) -> Tuple[int, int]:
    """This rank's contiguous range of the 2^32 erf bit patterns."""
    return split(SWEEP_PATTERNS, world, rank)


def sweep_chunks(lo: int, hi: int, chunk: int = 1 << 24) -> List[Tuple[int, int]]:
    """(base, count) pieces of [lo, hi), each at most `chunk` patterns."""
    return [(b, min(chunk, hi - b)) for b in range(lo, hi, chunk)]


def sum_over_ranks(dist, value: int) -> int:
    """Sum of one integer per rank (mismatch counts), on every rank."""
    if dist is None:
        return int(value)
    import torch
    t = torch.tensor([int(value)], dtype=torch.int64)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return int(t.item())


def max_over_ranks(dist, value: float) -> float:
    """Max of one float per rank (device times: the job ends with the slowest)."""
    if dist is None:
        return float(value)
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_rows(dist, local: np.ndarray, world: int, rank: int, root: int = 0):
    """Concatenate every rank's block of rows at `root`, in rank order (the one
    gather of results); other ranks get None. Blocks may differ in length."""
    if dist is None or world == 1:
        return local
    import torch
    n = torch.tensor([local.shape[0]], dtype=torch.int64)
    sizes = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(sizes, n)
    rows = [int(s.item()) for s in sizes]
    width = int(np.prod(local.shape[1:])) if local.ndim > 1 else 1
    pad = max(rows)
    buf = np.zeros((pad, width), dtype=local.dtype)
    buf[: local.shape[0]] = local.reshape(local.shape[0], width)
    t = torch.from_numpy(buf.view(np.uint8).copy())
    if rank == root:
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.gather(t, gather_list=parts, dst=root)
        out = [p.numpy().view(local.dtype).reshape(pad, width)[:r] for p, r in zip(parts, rows)]
        return np.concatenate(out, axis=0).reshape((sum(rows),) + local.shape[1:])
    dist.gather(t, dst=root)
    return None
