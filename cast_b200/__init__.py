"""cast_b200: B200-native ragged tree-verification attention and tree construction.

A drop-in for the hot path of CAST (js-lee-AI/CAST):
``cast_trees.tree_attn.varlen_tree_attention`` and the tree builder that feeds
it (``cast_trees.tree.block_topk`` / ``build_tree``). The compute runs in
hand-written sm_100a CUDA kernels behind a C ABI (include/cast_b200.h); this
package is the Python face of that library and has no CPU fallback.
"""
__version__ = "0.1.0"

from .tree import TreeNode, Trees, block_topk, block_topk_device, build_tree, build_trees
from .tree_attn import attention_plan, varlen_tree_attention, varlen_tree_attention_store, workspace_size

__all__ = ["TreeNode", "Trees", "block_topk", "block_topk_device", "build_tree", "build_trees",
           "varlen_tree_attention", "varlen_tree_attention_store", "workspace_size", "attention_plan",
           "__version__"]
