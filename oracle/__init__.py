"""CPU oracle for the ragged tree-verification path (TEST INFRASTRUCTURE ONLY).

This package restates, on the CPU, the reference algorithms that the CUDA
library in ``cast_b200`` replaces:

* ``oracle.tree``  - ``block_topk`` / ``build_tree`` / ``ancestor_matrix`` of
  cast_trees/tree.py:20-49,85-93, the pack bitmask recurrence of
  cast_trees/serving.py:213-222 and the greedy tree walk of
  cast_trees/decode.py:85-103, and ``select_global_topk`` of
  cast_trees/tree.py:63-82.
* ``oracle.kv``    - ``BatchedServer._append_store`` of
  cast_trees/serving.py:264-289 and ``gather_cache`` of
  cast_trees/verify.py:48-60.
* ``oracle.attn``  - the per-sequence fp32 dense masked softmax of
  tests/test_tree_attn.py:40-59 (equivalently cast_trees/verify.py:15-25 plus
  scaled-dot-product attention, as cast_trees/serving.py:52-54 calls it).

Parity is pinned: ``tests/golden/make_golden.py`` ran the reference package
itself and committed its outputs under ``tests/golden/``; the CPU test suite
checks this oracle against every one of them.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this package, and only as the checker or the timed
CPU baseline. The product path (``cast_b200``) never imports it.
"""
