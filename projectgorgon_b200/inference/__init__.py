"""Verifier and KV-cache operators under ProjectGorgon's names (``gorgon.inference``)."""
from .kv_cache import GorgonKVCache, apply_cache_slice
from .tree_candidates import (CandidateTree, CandidateTrees, HeadStatistics, build_candidate_tree,
                              build_candidate_trees, head_candidate_trees, head_statistics, max_tree_nodes,
                              medusa_head_inputs)
from .tree_decode import (TreeStepResult, gorgon_tree_attention, register_tree_attention, tree_forward,
                          tree_verify_step, trim_hf_cache)
from .verify import TreeVerifyResult, accept_draft_tokens, verify_tree

__all__ = ["GorgonKVCache", "apply_cache_slice", "TreeVerifyResult", "accept_draft_tokens",
           "verify_tree", "CandidateTree", "CandidateTrees", "HeadStatistics", "build_candidate_tree",
           "build_candidate_trees", "head_candidate_trees", "head_statistics", "max_tree_nodes",
           "medusa_head_inputs", "TreeStepResult",
           "gorgon_tree_attention", "register_tree_attention", "tree_forward", "tree_verify_step", "trim_hf_cache"]
