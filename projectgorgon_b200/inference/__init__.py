"""Verifier and KV-cache operators under ProjectGorgon's names (``gorgon.inference``)."""
from .kv_cache import GorgonKVCache, apply_cache_slice
from .tree_candidates import (CandidateTree, CandidateTrees, HeadStatistics, build_candidate_tree,
                              build_candidate_trees, head_statistics, max_tree_nodes)
from .verify import TreeVerifyResult, accept_draft_tokens, verify_tree

__all__ = ["GorgonKVCache", "apply_cache_slice", "TreeVerifyResult", "accept_draft_tokens",
           "verify_tree", "CandidateTree", "CandidateTrees", "HeadStatistics", "build_candidate_tree",
           "build_candidate_trees", "head_statistics", "max_tree_nodes"]
