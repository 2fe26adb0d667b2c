"""The bounded-wait failure path of the tensor-core attention kernel, made to happen on purpose.

cast_test_set_wait_limit_ns shortens the kernel's pipeline waits (ring slots,
copies, MMAs, softmax hand-offs) far below the time one TMA copy takes, so the
first wait for the query tile runs out. The kernel must then report
CAST_DEV_TIMEOUT through the device error word, drain its in-flight copies and
MMAs under the full limit and return; nothing hangs or faults. A normal call on
the same GPU afterwards must still match the oracle.
"""
import numpy as np
import pytest
import torch

import cast_b200
from cast_b200 import _lib
from oracle import attn as oattn
from oracle import tree as otree

pytestmark = pytest.mark.gpu


def _case(dev):
    g = torch.Generator().manual_seed(11)
    rng = np.random.default_rng(11)
    S, P = [1500, 300, 0], [40, 100, 9]
    parents, cu_q, cu_kv = [], [0], [0]
    for s, p in zip(S, P):
        parents += [-1] + [int(rng.integers(0, i)) for i in range(1, p)]
        cu_q.append(cu_q[-1] + p)
        cu_kv.append(cu_kv[-1] + s + p)
    q = torch.randn(cu_q[-1], 32, 128, generator=g) * 0.5
    k = torch.randn(cu_kv[-1], 8, 128, generator=g) * 0.5
    v = torch.randn(cu_kv[-1], 8, 128, generator=g) * 0.5
    i32 = lambda x: torch.tensor(x, dtype=torch.int32, device=dev)
    args = (q.to(dev, torch.bfloat16), k.to(dev, torch.bfloat16), v.to(dev, torch.bfloat16), i32(cu_q), i32(cu_kv),
            i32(S), i32(P), None)
    words = [otree.ancestor_words(np.array(parents[cu_q[b]:cu_q[b + 1]], np.int32)) for b in range(len(S))]
    return args, i32(parents), (cu_q, cu_kv, S, P, words)


def test_pipeline_wait_runs_out_then_recovers(cuda):
    args, parent, meta = _case(cuda)
    q, k, v = args[:3]
    kernel, n_split, _ = cast_b200.attention_plan(q, k, v, torch.empty_like(q), 3, 100, 1540)
    assert kernel == "tcgen05" and n_split == 1
    L = _lib.lib()
    assert _lib.device_error() == 0
    L.cast_test_set_wait_limit_ns(200)        # 200 ns: shorter than any copy from HBM
    try:
        cast_b200.varlen_tree_attention(*args, parent=parent, max_pack=100, max_kv=1540)
        code = _lib.device_error()
    finally:
        L.cast_test_set_wait_limit_ns(0)
    assert code == _lib.CAST_DEV_TIMEOUT, code
    # the context is still usable and the default limit is back: a normal call matches the oracle
    out = cast_b200.varlen_tree_attention(*args, parent=parent, max_pack=100, max_kv=1540)
    assert _lib.device_error() == 0
    cu_q, cu_kv, S, P, words = meta
    expect = oattn.tree_attention(q.float().cpu(), k.float().cpu(), v.float().cpu(), cu_q, cu_kv, S, P, words)
    err = (out.float().cpu() - expect).abs().max().item()
    assert err < 2e-2, err
