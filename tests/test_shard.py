"""Token-balanced sequence partition and the pooled-embedding gather (CPU, Gloo ranks)."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from packed_encoders_b200 import shard
from packed_encoders_b200 import workloads as wl


def test_band_pairs_matches_oracle_counts():
    import oracle

    for n in (1, 2, 63, 64, 65, 130, 500):
        cu = torch.tensor([0, n], dtype=torch.int32)
        assert shard.band_pairs(n) == oracle.useful_pairs(cu)
        assert shard.band_pairs(n, (64, 64)) == oracle.useful_pairs(cu, window=(64, 64))
        assert shard.band_pairs(n, causal=True) == oracle.useful_pairs(cu, causal=True)
        assert shard.band_pairs(n, (8, -1), causal=True) == oracle.useful_pairs(cu, window=(8, -1), causal=True)


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_partition_covers_every_sequence_once_and_balances(world):
    lengths = wl.config3_lengths(512 * world, seed=0)
    costs = [shard.pattern_cost(n, (wl.GLOBAL, wl.LOCAL64), alpha=64.0) for n in lengths]
    shards = shard.partition(lengths, world, costs)
    assert [s.rank for s in shards] == list(range(world))
    seen = sorted(i for s in shards for i in s.indices)
    assert seen == list(range(len(lengths)))
    for s in shards:
        assert list(s.indices) == sorted(s.indices)
        assert s.lengths == tuple(lengths[i] for i in s.indices)
        assert s.cu_seqlens()[-1].item() == s.tokens
    loads = [s.load for s in shards]
    # LPT: no rank exceeds the mean by more than the largest single job
    assert max(loads) - sum(loads) / world <= max(costs) + 1e-6
    assert shard.partition(lengths, world, costs) == shards  # deterministic


def test_partition_edge_cases():
    assert [s.lengths for s in shard.partition([], 2)] == [(), ()]
    s = shard.partition([5, 0, 3], 4)
    assert sum(len(x.indices) for x in s) == 3
    with pytest.raises(ValueError):
        shard.partition([1, 2], 0)


def _free_port() -> int:
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def _gather_worker(rank, world, port, lengths, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shards = shard.partition(lengths, world)
        mine = shards[rank]
        pooled = torch.tensor([[float(i), float(lengths[i])] for i in mine.indices]).reshape(-1, 2)
        out = shard.gather_pooled(pooled, mine, shards)
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_gather_pooled_restores_original_order_over_gloo():
    world = 2
    lengths = [5, 900, 17, 3, 300, 41, 1, 2, 64]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, world, port, lengths, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    expected = torch.tensor([[float(i), float(n)] for i, n in enumerate(lengths)])
    for rank in range(world):
        assert torch.equal(results[rank], expected)


def _dead_rank_worker(rank, world, port, q):
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    try:
        if rank == 1:
            raise RuntimeError("rank 1 fails before the gather")
        lengths = [4, 8, 15, 16]
        shards = shard.partition(lengths, world)
        shard.gather_pooled(torch.zeros(len(shards[0].indices), 2), shards[0], shards)
        q.put((rank, "completed"))
    except RuntimeError as exc:
        q.put((rank, f"error: {type(exc).__name__}"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def test_a_failing_rank_surfaces_as_an_error_not_a_hang():
    """A rank that raises before the collective: the survivor's gather ends with an error once
    the short process-group timeout passes (no GPU involved)."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dead_rank_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert results[1].startswith("error")
    assert results[0].startswith("error")
