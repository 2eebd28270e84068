"""The multi-rank host logic on CPU, over ``gloo`` ranks (spawned processes,
rendezvous on 127.0.0.1): the max-of-times / sum-of-work reduction of bench.py,
the (sequence, head) → rank assignment of the op's head sharding, and the
reassembly of O along heads (the oracle's forward on each rank's heads,
all-gathered, equals the oracle's forward on the whole batch)."""

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


def _shard_worker(rank: int, world: int, port: int, out_dir: str) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import numpy as np
    import torch
    import torch.distributed as dist
    from dsalt.kernels.head_shard import gather_heads, reduce_window_grad, shard_op_inputs
    from oracle import dsalt_oracle as O
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        inp = _global_batch()
        sh = shard_op_inputs(inp["q"], inp["k"], inp["v"], inp["pos"], inp["logw"], rank, world,
                             extra={"do": inp["do"]})
        o, _ = O.attention_fwd(sh["q"].numpy(), sh["k"].numpy(), sh["v"].numpy(), sh["lmk_pos"].numpy(),
                               sh["lmk_logw"].numpy(), inp["w"].numpy(), inp["cu"].numpy())
        full = gather_heads(torch.from_numpy(np.ascontiguousarray(o)), inp["q"].shape[1])
        g = O.attention_bwd(sh["q"].numpy(), sh["k"].numpy(), sh["v"].numpy(), sh["do"].numpy(),
                            sh["lmk_pos"].numpy(), sh["lmk_logw"].numpy(), inp["w"].numpy(), inp["cu"].numpy(),
                            1.0, 4.0, "train")
        d_w = reduce_window_grad(torch.from_numpy(np.ascontiguousarray(g["d_w"])))
        torch.save({"heads": sh["heads"], "o": full, "d_w": d_w}, os.path.join(out_dir, f"shard{rank}.pt"))
    finally:
        dist.destroy_process_group()


def _global_batch():
    import torch
    g = torch.Generator().manual_seed(11)
    lens, H, D, k = [70, 45, 90], 5, 16, 6
    T = sum(lens)
    q, kk, v = (torch.randn(T, H, D, generator=g, dtype=torch.float64) for _ in range(3))
    w = 2 + torch.rand(T, generator=g, dtype=torch.float64) * 30
    pos = torch.stack([torch.stack([torch.randperm(L, generator=g)[:k] for L in lens]) for _ in range(H)])
    logw = torch.log(torch.sigmoid(torch.randn(H, len(lens), k, generator=g, dtype=torch.float64)))
    cu = torch.tensor([0, 70, 115, 205], dtype=torch.int32)
    do = torch.randn(T, H, D, generator=g, dtype=torch.float64)
    return dict(q=q, k=kk, v=v, w=w, pos=pos, logw=logw, cu=cu, do=do)


@pytest.mark.parametrize("world", [2, 3])
def test_head_shards_reassemble_to_the_whole_op(tmp_path, world):
    """5 heads over 2 or 3 ranks (uneven shards): every rank's all-gathered O equals
    the oracle's forward over all heads at once, and the all-reduced shard sums of
    ∂loss/∂w̃ equal the oracle's gradient over all heads."""
    import numpy as np
    import torch
    from oracle import dsalt_oracle as O
    mp.spawn(_shard_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    inp = _global_batch()
    ref, _ = O.attention_fwd(inp["q"].numpy(), inp["k"].numpy(), inp["v"].numpy(), inp["pos"].numpy(),
                             inp["logw"].numpy(), inp["w"].numpy(), inp["cu"].numpy())
    g = O.attention_bwd(inp["q"].numpy(), inp["k"].numpy(), inp["v"].numpy(), inp["do"].numpy(), inp["pos"].numpy(),
                        inp["logw"].numpy(), inp["w"].numpy(), inp["cu"].numpy(), 1.0, 4.0, "train")
    covered = []
    for r in range(world):
        got = torch.load(tmp_path / f"shard{r}.pt")
        covered.append(tuple(got["heads"]))
        assert np.array_equal(got["o"].numpy(), ref)
        assert np.allclose(got["d_w"].numpy(), g["d_w"], rtol=1e-5, atol=1e-6)
    assert covered[0][0] == 0 and covered[-1][1] == 5
    assert all(a[1] == b[0] for a, b in zip(covered, covered[1:]))


@pytest.mark.parametrize("world,per_rank", [(1, 16), (2, 8), (4, 4), (8, 2)])
def test_config2_units_per_rank(world, per_rank):
    """Config 2's 64 (sequence, head) units: 4 sequences × 16 heads split by heads,
    8 units per GPU at N = 8; contiguous, disjoint, covering every head."""
    from dsalt.kernels.head_shard import head_range
    ranges = [head_range(16, world, r) for r in range(world)]
    assert all(h1 - h0 == per_rank for h0, h1 in ranges)
    assert ranges[0][0] == 0 and ranges[-1][1] == 16
    assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
    assert 4 * per_rank * world == 64


def test_head_range_uneven_and_invalid():
    from dsalt.kernels.head_shard import head_range
    assert [head_range(5, 3, r) for r in range(3)] == [(0, 2), (2, 4), (4, 5)]
    with pytest.raises(ValueError):
        head_range(2, 4, 0)
    with pytest.raises(ValueError):
        head_range(8, 2, 2)
