"""Multi-rank host logic of the batch-sharded benchmark, on CPU with gloo
(world size 2): shards cover the global batch exactly once, the timing
reduction returns the slowest rank, and a rank that fails before the
collective is seen by the others as an error within the group timeout."""

from __future__ import annotations

import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import pytest
import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parent.parent


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def worker(rank: int, world: int, port: int, results, mode: str) -> None:
    sys.path.insert(0, str(REPO))
    import torch.distributed as dist

    import bench

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    try:
        if mode == "fail" and rank == 1:
            raise RuntimeError("rank 1 failed before the collective")
        start, count = bench.shard(1000, world, rank)
        slowest = bench.max_over_ranks(10.0 + rank, world)
        bench.barrier(world)
        results[rank] = (start, count, slowest)
    except Exception as error:  # reported to the parent, never hangs
        results[rank] = ("error", type(error).__name__)
    finally:
        if mode != "fail":
            dist.destroy_process_group()


def run(world: int, mode: str) -> dict:
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, world, port, results, mode)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank did not finish")
    return dict(results)


def test_shards_and_max_reduction_two_ranks():
    results = run(2, "ok")
    assert results[0] == (0, 500, 11.0)
    assert results[1] == (500, 500, 11.0)


def test_shard_plan_covers_batch_exactly_once():
    sys.path.insert(0, str(REPO))
    import bench

    for total in (1, 7, 256, 2048, 1001):
        for world in (1, 2, 3, 4, 8):
            covered = []
            for rank in range(world):
                start, count = bench.shard(total, world, rank)
                covered.extend(range(start, start + count))
            assert covered == list(range(total))


def test_failed_rank_surfaces_as_error_not_hang():
    results = run(2, "fail")
    assert results[1][0] == "error"
    assert results[0][0] == "error"  # the survivor's collective times out
