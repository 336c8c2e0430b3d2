"""B200-native (sm_100a) tree-verification path of speculative decoding.

The operators keep ProjectGorgon's Python names and arguments:

* ``build_tree_mask``, ``tree_attention`` (``tree_attention_cuda`` /
  ``tree_attention_triton``), ``fused_tree_verify``       -- ``kernels``
* ``verify_tree``, ``accept_draft_tokens``, ``apply_cache_slice``,
  ``GorgonKVCache.trim``, ``build_candidate_tree``          -- ``inference``

Every operator runs in ``lib/libgorgon_b200.so`` (hand-written CUDA for
sm_100a behind a C ABI, ``include/gorgon_b200.h``).  Host tensors raise
``ValueError``; a missing library raises ``ImportError`` on first use.
"""
from . import _abi
from .inference import (CandidateTree, GorgonKVCache, TreeVerifyResult, accept_draft_tokens, apply_cache_slice,
                        build_candidate_tree, build_candidate_trees, head_statistics, verify_tree)
from .kernels import (build_tree_mask, candidate_tree_to_mask, fused_tree_verify, tree_attention,
                      tree_attention_cuda, tree_attention_plan, tree_attention_triton)

__all__ = [
    "build_tree_mask", "candidate_tree_to_mask", "tree_attention", "tree_attention_plan", "tree_attention_cuda",
    "tree_attention_triton", "fused_tree_verify", "verify_tree", "accept_draft_tokens",
    "apply_cache_slice", "GorgonKVCache", "TreeVerifyResult", "device_error", "load_library",
    "CandidateTree", "build_candidate_tree", "build_candidate_trees", "head_statistics",
]


def load_library():
    """Loads the CUDA library now (it is otherwise loaded on first use)."""
    return _abi.lib()


def device_error(clear: bool = True) -> int:
    """Synchronously reads the library's device error bits (see gorgon_b200.h)."""
    return _abi.device_error(clear)
