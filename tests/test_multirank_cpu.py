"""The multi-rank host logic of bench.py on CPU: two ``gloo`` ranks (spawned
processes, rendezvous on 127.0.0.1) take the max of the timed milliseconds and the
sum of the work exactly as the GPU runs do over NCCL; config 5's head sharding."""

from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out_dir: str) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist
    import bench
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        # rank r timed 1 + r ms and did 10·(r + 1) units of work
        ms, work = bench.job_totals(1.0 + rank, 10.0 * (rank + 1), world, "cpu")
        with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
            f.write(f"{ms} {work}")
    finally:
        dist.destroy_process_group()


def test_job_totals_over_two_gloo_ranks(tmp_path):
    world = 2
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        ms, work = map(float, (tmp_path / f"rank{r}.txt").read_text().split())
        assert ms == 2.0            # the slowest rank's time
        assert work == 30.0         # the whole job's work


def test_single_rank_totals_pass_through():
    import bench
    assert bench.job_totals(3.5, 7.0, 1, "cpu") == (3.5, 7.0)


@pytest.mark.parametrize("world,heads", [(1, 32), (2, 16), (4, 8), (8, 4)])
def test_config5_head_shards(world, heads):
    import bench
    assert bench.config5_shard(world) == heads
    assert heads * world == bench.CONFIG5["H"]


def test_config5_rejects_uneven_shards():
    import bench
    with pytest.raises(SystemExit):
        bench.config5_shard(3)
