"""The multi-GPU plumbing of bench.py on CPU: two gloo ranks (world size 2)
run the same partition, barrier, max-over-ranks and gather logic the GPU
ranks run over NCCL. Sequences are independent, so the data path has no
collective: each rank owns a contiguous range of the global batch."""
from __future__ import annotations

import os
import sys

import pytest

from conftest import REPO

torch = pytest.importorskip("torch")
mp = pytest.importorskip("torch.multiprocessing")


def _rank_main(rank, world, port, q):
    os.environ.update({"RANK": str(rank), "LOCAL_RANK": str(rank), "WORLD_SIZE": str(world),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    sys.path.insert(0, str(REPO))
    import bench
    d = bench.Dist(backend="gloo", cuda=False)
    d.init(torch)
    try:
        total = 1024
        start, count = bench.shard(total, world, rank)
        d.barrier(torch)
        # each rank "steps" its own sequences: fake per-rank timings and tokens
        ms = d.max(torch, 1.0 + rank)
        owned = d.gather(torch, [start, count])
        sums = d.gather(torch, [sum(range(start, start + count))])
        q.put((rank, ms, owned, sums))
    finally:
        d.close()


def test_two_gloo_ranks_partition_max_and_gather():
    port = 29500 + (os.getpid() % 1000)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ms, owned, sums in res:
        assert ms == 2.0  # the slower rank's time, on every rank
        assert owned == [[0.0, 512.0], [512.0, 512.0]]
        assert sum(s[0] for s in sums) == sum(range(1024))  # every sequence exactly once


@pytest.mark.parametrize("total,world", [(1024, 1), (1024, 2), (1024, 8), (64, 8), (10, 4),
                                         (3, 8)])
def test_shard_covers_the_batch_once(total, world):
    import bench
    seen = []
    for r in range(world):
        s, c = bench.shard(total, world, r)
        seen += list(range(s, s + c))
        assert abs(c - total / world) < 1
    assert seen == list(range(total))
