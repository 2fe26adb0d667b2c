"""Host logic of the multi-GPU split: LPT sequence shards, checked on CPU and
across two gloo ranks (world_size 2), with no GPU."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cast_b200 import sharding, workloads


def test_lpt_covers_every_sequence_once():
    w = workloads.config(5)
    for world in (1, 2, 4, 8):
        shards = sharding.lpt_shards([sharding.sequence_cost(s, p) for s, p in zip(w.S, w.P)], world)
        flat = sorted(i for sh in shards for i in sh)
        assert flat == list(range(w.B))
        assert sharding.imbalance(w.S, w.P, shards) < 1.01      # 512 ragged sequences balance well


def test_lpt_small_cases():
    assert sharding.lpt_shards([5, 1, 1, 1, 1, 1], 2) == [[0], [1, 2, 3, 4, 5]]
    assert sharding.lpt_shards([], 3) == [[], [], []]
    with pytest.raises(ValueError):
        sharding.lpt_shards([1], 0)


def test_equal_count_shards_balance_the_weak_scaling_batch():
    # 64 sequences per GPU of the configuration-3 recipe, drawn as one batch of 64 * world
    for world in (1, 2, 4, 8):
        S, N = workloads._ragged(2, 64 * world, 4096, 8192, (127,))
        costs = [sharding.sequence_cost(s, n + 1) for s, n in zip(S, N)]
        shards = sharding.equal_count_shards(costs, world, 64)
        assert all(len(sh) == 64 for sh in shards)
        assert sorted(i for sh in shards for i in sh) == list(range(64 * world))
        loads = [sum(costs[i] for i in sh) for sh in shards]
        assert max(loads) / (sum(loads) / world) < 1.002
    assert sharding.equal_count_shards([9, 1, 8, 2], 2, 2) == [[0, 1], [2, 3]]
    with pytest.raises(ValueError):
        sharding.equal_count_shards([1, 2, 3], 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    w = workloads.config(2)
    mine = sharding.shard_of(w.S, w.P, rank, world)
    sub = w.shard(mine)
    # every rank's shard keeps the global sequence ids and lengths
    assert sub.ids() == mine and sub.S == [w.S[i] for i in mine]
    gathered = [None] * world
    dist.all_gather_object(gathered, mine)
    cost = torch.tensor([float(sum(sharding.sequence_cost(w.S[i], w.P[i]) for i in mine))])
    dist.all_reduce(cost, op=dist.ReduceOp.MAX)
    if rank == 0:
        result.put((gathered, cost.item()))
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_partition_the_batch():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    gathered, max_cost = q.get(timeout=120)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    w = workloads.config(2)
    assert sorted(gathered[0] + gathered[1]) == list(range(w.B))
    assert not set(gathered[0]) & set(gathered[1])
    total = sum(sharding.sequence_cost(s, p) for s, p in zip(w.S, w.P))
    assert max_cost <= 0.6 * total
