"""The Python host layer without a GPU: every entry point refuses CPU tensors
loudly (there is no CPU fallback) and checks its arguments before the C ABI."""
import types

import numpy as np
import pytest
import torch

import cast_b200


def test_attention_refuses_cpu_tensors():
    q = torch.zeros(4, 8, 128)
    k = torch.zeros(8, 2, 128)
    i32 = lambda x: torch.tensor(x, dtype=torch.int32)
    with pytest.raises(RuntimeError, match="CUDA"):
        cast_b200.varlen_tree_attention(q, k, k, i32([0, 4]), i32([0, 8]), i32([4]), i32([4]), None,
                                        parent=i32([-1, 0, 1, 2]))
    with pytest.raises(RuntimeError, match="CUDA"):
        cast_b200.varlen_tree_attention_store(q, k[None].transpose(1, 2), k[None].transpose(1, 2), k[:4], k[:4],
                                              i32([0, 4]), i32([4]), i32([4]), None, parent=i32([-1, 0, 1, 2]))


def test_walk_refuses_cpu_tensors():
    with pytest.raises(RuntimeError, match="CUDA"):
        cast_b200.walk_trees_greedy(torch.zeros(3, 10), torch.tensor([0, 3]), [-1, 0, 1], [1, 2, 3], 2)


def test_walk_tree_temperature_above_zero_is_not_supported():
    with pytest.raises(NotImplementedError):
        cast_b200.walk_tree([], torch.zeros(1, 4), temperature=0.7)


def test_store_append_and_gather_refuse_cpu_tensors():
    buf = [torch.zeros(2, 2, 8, 16)]
    pack = [torch.zeros(2, 5, 16)]
    with pytest.raises(RuntimeError, match="CUDA"):
        cast_b200.append_store(buf, buf, [1, 2], [0, 2, 5], [[0], [0, 1]], [1, 2], [0, 1], pack, pack)
    cache = types.SimpleNamespace(key_cache=[torch.zeros(1, 2, 8, 16)], value_cache=[torch.zeros(1, 2, 8, 16)])
    with pytest.raises(RuntimeError, match="CUDA"):
        cast_b200.gather_cache(cache, 4, [0, 2])


def test_cache_layers_handles_both_layouts():
    old = types.SimpleNamespace(key_cache=[1, 2], value_cache=[3, 4])
    n, get, put = cast_b200.cache_layers(old)
    assert n == 2 and get(1) == (2, 4)
    put(0, 5, 6)
    assert old.key_cache[0] == 5 and old.value_cache[0] == 6
    new = types.SimpleNamespace(layers=[types.SimpleNamespace(keys=7, values=8)])
    n, get, put = cast_b200.cache_layers(new)
    assert n == 1 and get(0) == (7, 8)


def test_select_global_topk_of_no_trees_is_empty():
    assert cast_b200.select_global_topk([], 10) == []


def test_ancestor_bits_match_the_oracle_words():
    # the int64 word the reference's Triton kernel takes, built on the torch side for the head-to-head
    import numpy as np
    import torch
    from cast_b200.bench_case import _ancestor_bits
    from oracle import tree as otree
    rng = np.random.default_rng(5)
    parents, cu = [], [0]
    for P in (1, 17, 64, 33):
        par = [-1] + [int(rng.integers(max(0, i - 5), i)) for i in range(1, P)]
        parents += par
        cu.append(cu[-1] + P)
    pp = torch.tensor(parents, dtype=torch.int32)
    cu_q = torch.tensor(cu, dtype=torch.int32)
    got = _ancestor_bits(pp, cu_q, cu_q[1:] - cu_q[:-1], 64).numpy()
    want = np.concatenate([otree.ancestor_words(np.array(parents[cu[b]:cu[b + 1]], np.int32)).reshape(-1)
                           for b in range(4)]).view(np.int64)
    assert np.array_equal(got, want)
