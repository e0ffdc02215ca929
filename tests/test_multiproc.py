"""Multi-rank host logic on CPU with gloo, world_size 2: sample sharding, the max-over-ranks
timing reduction used by bench.py, and host-side failure detection (a rank that raises, a
rank that never joins)."""
import datetime
import time

import pytest

from lithe_b200.shard import RankFailure, imbalance, run_ranks, shard_bounds, shard_sizes


def test_shard_sizes():
    assert shard_sizes(14, 8) == [2, 2, 2, 2, 2, 2, 1, 1]
    assert shard_sizes(14, 1) == [14]
    assert shard_sizes(3, 4) == [1, 1, 1, 0]
    assert [shard_bounds(14, 4, r) for r in range(4)] == [(0, 4), (4, 8), (8, 11), (11, 14)]
    assert sum(shard_sizes(96, 8)) == 96 and imbalance(14, 8) == pytest.approx(2 / 1.75)
    with pytest.raises(ValueError):
        shard_bounds(4, 2, 2)


def _init(world):
    import torch.distributed as dist
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=20))
    return dist


def _max_and_gather(rank, world):
    import torch
    dist = _init(world)
    # what each rank would time and own
    t = torch.tensor([10.0 + 5.0 * rank], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    start, end = shard_bounds(14, world, rank)
    owned = torch.tensor([start, end], dtype=torch.int64)
    got = [torch.zeros(2, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(got, owned)
    dist.barrier()
    dist.destroy_process_group()
    return float(t.item()), [tuple(g.tolist()) for g in got]


def test_max_over_ranks_and_shards_gloo():
    res = run_ranks(_max_and_gather, 2, timeout=120)
    assert [r[0] for r in res] == [15.0, 15.0]
    assert res[0][1] == [(0, 7), (7, 14)] and res[1][1] == res[0][1]


def _one_raises(rank, world):
    dist = _init(world)
    if rank == 1:
        raise RuntimeError("injected failure on rank 1")
    dist.barrier()          # rank 0 blocks here until the parent stops it
    return rank


def test_rank_exception_is_reported():
    t0 = time.monotonic()
    with pytest.raises(RankFailure) as ei:
        run_ranks(_one_raises, 2, timeout=60)
    assert 1 in ei.value.failures and "injected failure on rank 1" in ei.value.failures[1]
    assert time.monotonic() - t0 < 50


def _never_joins(rank, world):
    if rank == 1:
        time.sleep(3600)
    dist = _init(world)
    dist.barrier()
    return rank


def test_hung_rank_is_detected_by_deadline():
    t0 = time.monotonic()
    with pytest.raises(RankFailure) as ei:
        run_ranks(_never_joins, 2, timeout=8)
    assert 1 in ei.value.failures
    assert time.monotonic() - t0 < 40
