"""Sequence sharding of a verify batch over GPUs (no collective on the path).

Sequences of a ragged verify batch are independent (each reads only its own
prefix and pack, cast_trees/tree_attn.py:39-41), so a batch splits across GPUs
by whole sequences. The cost of a sequence is P_b * (S_b + P_b), proportional
to both its attention flops and its K/V bytes; the longest-processing-time
rule (largest cost first, onto the least-loaded GPU) balances the shards.
"""
import heapq


def sequence_cost(prefix_len, pack_len):
    return int(pack_len) * (int(prefix_len) + int(pack_len))


def lpt_shards(costs, n_shards):
    """Index lists per shard; each list is sorted ascending (pack order kept)."""
    if n_shards < 1:
        raise ValueError("n_shards must be >= 1")
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    heap = [(0, s) for s in range(n_shards)]
    shards = [[] for _ in range(n_shards)]
    for i in order:
        load, s = heapq.heappop(heap)
        shards[s].append(i)
        heapq.heappush(heap, (load + costs[i], s))
    return [sorted(x) for x in shards]


def equal_count_shards(costs, n_shards, per_shard):
    """LPT with a cardinality cap: exactly `per_shard` indices per shard.

    For weak scaling the per-GPU batch size is fixed; the largest cost goes
    first onto the least-loaded shard that still has room. Needs
    len(costs) == n_shards * per_shard. Each list is sorted ascending.
    """
    if n_shards < 1 or per_shard < 0 or len(costs) != n_shards * per_shard:
        raise ValueError("need n_shards >= 1 and len(costs) == n_shards * per_shard")
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    heap = [(0, s) for s in range(n_shards)]
    shards = [[] for _ in range(n_shards)]
    for i in order:
        load, s = heapq.heappop(heap)
        shards[s].append(i)
        if len(shards[s]) < per_shard:
            heapq.heappush(heap, (load + costs[i], s))
    return [sorted(x) for x in shards]


def shard_of(prefix_len, pack_len, rank, world):
    """Sequence indices this rank processes."""
    costs = [sequence_cost(s, p) for s, p in zip(prefix_len, pack_len)]
    return lpt_shards(costs, world)[rank]


def imbalance(prefix_len, pack_len, shards):
    """max shard cost / mean shard cost (1.0 = perfect)."""
    costs = [sequence_cost(s, p) for s, p in zip(prefix_len, pack_len)]
    loads = [sum(costs[i] for i in sh) for sh in shards]
    mean = sum(loads) / len(loads)
    return max(loads) / mean if mean > 0 else 1.0
