"""Both 16-bit tensor-core attention kernels against the CPU oracle and each other (GPU).

Regular-layout bf16/fp16 calls whose largest head group fills whole 256-row pairs run the CTA-pair
kernel (tcgen05 cta_group::2: a 256-row block over the two SMs of a TPC, three S buffers per SM);
the others, and store mode, run the single-CTA kernel (two 128-row query tiles per SM). The test
hook cast_test_set_tc_kernel(0) forces the single-CTA kernel; the cases below put each shape through
both where the pair applies: one to many key tiles, S = 0, P = 1, ragged batches, G from 1 to 16,
a 260-row head group (and long ones split between a pair launch and a single-CTA launch), split
keys, and batches of more sequences than the kernels rank by length.
"pair" cases have G * max_pack a multiple of 256.
"""
import numpy as np
import pytest
import torch

import cast_b200
from cast_b200 import _lib
from oracle import attn as oattn
from oracle import tree as otree

pytestmark = pytest.mark.gpu

CASES = [
    ("pair one tile", [100], [64], 32, 8),
    ("pair ragged", [0, 129, 256, 1000, 4000, 37], [1, 64, 128, 127, 65, 128], 32, 8),
    ("pair P=1 neighbour", [700, 300], [1, 128], 32, 8),
    ("pair G=1", [500, 300], [100, 256], 8, 8),
    ("pair G=16", [900, 64], [64, 16], 128, 8),
    ("pair split keys", [20000, 15000], [128, 100], 32, 8),
    # more sequences than the kernels rank by length (they then run in sequence order)
    ("pair 160 sequences", [int(x) for x in np.random.default_rng(3).integers(0, 400, 160)],
     [64] + [int(x) for x in np.random.default_rng(4).integers(1, 65, 159)], 32, 8),
    ("one tile", [100], [20], 32, 8),
    ("two tiles", [200], [30], 32, 8),
    ("many tiles", [3000], [64], 32, 8),
    ("no prefix", [0], [50], 32, 8),
    ("one token", [700], [1], 32, 8),
    ("ragged", [0, 129, 256, 1000, 4000, 37], [1, 64, 128, 127, 65, 200], 32, 8),
    ("G=1", [500, 300], [100, 300], 8, 8),
    ("G=2", [500, 1300], [100, 300], 16, 8),
    ("G=8", [500, 1300], [100, 33], 64, 8),
    ("G=16", [900, 64], [70, 16], 128, 8),
    ("260 rows", [2000], [65], 32, 8),
    # long units ending in a one-tile block: full 256-row blocks on CTA pairs, the last blocks on single CTAs
    ("mixed pair and tail launches", [8192 + 37 * i for i in range(20)], [65] * 19 + [40], 32, 8),
    ("split keys", [20000, 15000], [128, 100], 32, 8),
    ("160 sequences", [int(x) for x in np.random.default_rng(5).integers(0, 400, 160)],
     [int(x) for x in np.random.default_rng(6).integers(1, 50, 160)], 32, 8),
]


def _case(S_list, P_list, Hq, Hkv, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    cu_q, cu_kv, par = [0], [0], []
    for S, P in zip(S_list, P_list):
        cu_q.append(cu_q[-1] + P)
        cu_kv.append(cu_kv[-1] + S + P)
        par += [-1] + [int(torch.randint(0, i, (1,), generator=g)) for i in range(1, P)]
    q = (torch.randn(cu_q[-1], Hq, 128, generator=g) * 0.5).to(dtype)
    k = (torch.randn(cu_kv[-1], Hkv, 128, generator=g) * 0.5).to(dtype)
    v = (torch.randn(cu_kv[-1], Hkv, 128, generator=g) * 0.5).to(dtype)
    return q, k, v, np.array(cu_q, np.int32), np.array(cu_kv, np.int32), np.array(S_list, np.int32), \
        np.array(P_list, np.int32), np.array(par, np.int32)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("name, S, P, Hq, Hkv", CASES)
def test_pair_and_single_kernels_match_oracle(cuda, name, S, P, Hq, Hkv, dtype):
    q, k, v, cu_q, cu_kv, S_, P_, par = _case(S, P, Hq, Hkv, dtype, sum(map(ord, name)))
    words = [otree.ancestor_words(par[cu_q[b]:cu_q[b + 1]]) for b in range(len(S))]
    expect = oattn.tree_attention(q.float(), k.float(), v.float(), cu_q, cu_kv, S_, P_, words)
    t = lambda a: torch.from_numpy(a).to(cuda)
    qd, kd, vd = q.to(cuda), k.to(cuda), v.to(cuda)
    assert cast_b200.attention_plan(qd, kd, vd, qd, len(S), int(P_.max()), int((S_ + P_).max()))[0] == "tcgen05"
    outs = {}
    L = _lib.lib()
    try:
        for kernel in (1, 0):
            L.cast_test_set_tc_kernel(kernel)
            outs[kernel] = cast_b200.varlen_tree_attention(qd, kd, vd, t(cu_q), t(cu_kv), t(S_), t(P_), None,
                                                           parent=t(par)).float().cpu()
            torch.cuda.synchronize()
            assert _lib.device_error() == 0
    finally:
        L.cast_test_set_tc_kernel(1)
    for kernel, out in outs.items():
        err = (out - expect).abs().max().item()
        assert err < 2e-2, (kernel, err)
    assert (outs[1] - outs[0]).abs().max().item() < 2e-2


@pytest.mark.parametrize("kernel", [1, 0])
def test_bad_metadata_is_reported_by_both_kernels(cuda, kernel):
    # pair-eligible shape (4 heads per KV head x 64-token packs = 256 rows): a parent that is not in
    # pack order, then a pack longer than the max_pack the caller promised. Both are recorded in the
    # device error word, nothing hangs or faults, and the next good call on the context is correct.
    q, k, v, cu_q, cu_kv, S_, P_, par = _case([300, 700], [64, 64], 32, 8, torch.bfloat16, 21)
    t = lambda a: torch.from_numpy(a).to(cuda)
    qd, kd, vd = q.to(cuda), k.to(cuda), v.to(cuda)
    L = _lib.lib()
    try:
        L.cast_test_set_tc_kernel(kernel)
        bad = par.copy()
        bad[cu_q[1] + 5] = 9                          # token 5 of the second pack: parent after itself
        cast_b200.varlen_tree_attention(qd, kd, vd, t(cu_q), t(cu_kv), t(S_), t(P_), None, parent=t(bad))
        assert _lib.device_error() == _lib.CAST_DEV_BAD_PARENT
        cast_b200.varlen_tree_attention(qd, kd, vd, t(cu_q), t(cu_kv), t(S_), t(P_), None, parent=t(par),
                                        max_pack=32, max_kv=int((S_ + P_).max()))
        assert _lib.device_error() == _lib.CAST_DEV_BAD_LAYOUT
        out = cast_b200.varlen_tree_attention(qd, kd, vd, t(cu_q), t(cu_kv), t(S_), t(P_), None, parent=t(par))
        assert _lib.device_error() == 0
    finally:
        L.cast_test_set_tc_kernel(1)
    words = [otree.ancestor_words(par[cu_q[b]:cu_q[b + 1]]) for b in range(2)]
    expect = oattn.tree_attention(q.float(), k.float(), v.float(), cu_q, cu_kv, S_, P_, words)
    assert (out.float().cpu() - expect).abs().max().item() < 2e-2
