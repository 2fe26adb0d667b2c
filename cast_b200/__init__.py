"""cast_b200: B200-native ragged tree-verification attention and tree construction.

A drop-in for the hot path of CAST (js-lee-AI/CAST):
``cast_trees.tree_attn.varlen_tree_attention`` and the tree builder that feeds
it (``cast_trees.tree.block_topk`` / ``build_tree``), plus the verify-round
steps around it: the greedy tree walk, ``select_global_topk`` and the KV-store
append / cache gather. The compute runs in
hand-written sm_100a CUDA kernels behind a C ABI (include/cast_b200.h); this
package is the Python face of that library and has no CPU fallback.
"""
__version__ = "0.1.0"

from .decode import Walk, walk_tree, walk_trees_greedy
from .serving import append_store, append_store_inplace
from .tree import (TreeNode, Trees, block_topk, block_topk_device, build_tree, build_trees, select_global_topk,
                   select_global_topk_device)
from .tree_attn import attention_plan, varlen_tree_attention, varlen_tree_attention_store, workspace_size

from .verify import cache_layers, gather_cache

__all__ = ["TreeNode", "Trees", "block_topk", "block_topk_device", "build_tree", "build_trees",
           "select_global_topk", "select_global_topk_device", "Walk", "walk_tree", "walk_trees_greedy",
           "append_store", "append_store_inplace", "cache_layers", "gather_cache",
           "varlen_tree_attention", "varlen_tree_attention_store", "workspace_size", "attention_plan",
           "__version__"]
