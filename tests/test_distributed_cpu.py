"""The bench's multi-rank glue on 2 gloo ranks (CPU only): slowest-rank
timing and the full-sum partial combine, the path's one collective."""

from __future__ import annotations

import os
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import REPO


def _worker(rank: int, world: int, port: int, q) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    sys.path.insert(0, str(REPO))
    import bench
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        slow = bench.max_over_ranks(1.0 + rank, world, "cpu")
        part = torch.tensor([float(rank + 1) * 10.0])
        bench.combine_step("c4", {"sum_1": part}, world)()
        untouched = torch.tensor([3.0])
        bench.combine_step("c2", {"sum_1": untouched}, world)()
        q.put((rank, slow, float(part.item()), float(untouched.item())))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    got = sorted(q.get(timeout=10) for _ in range(2))
    for rank, slow, total, untouched in got:
        assert slow == 2.0            # max over ranks
        assert total == 30.0          # 10 + 20: the partials are summed
        assert untouched == 3.0       # no collective for the sharded configs
