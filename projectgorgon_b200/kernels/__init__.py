"""Tree-verification operators under ProjectGorgon's names (``gorgon.kernels``)."""
from .fused_tree_verify_triton import fused_tree_verify
from .tree_attention import tree_attention, tree_attention_plan
from .tree_attention_cuda import tree_attention_cuda
from .tree_attention_triton import tree_attention_triton
from .tree_mask import build_tree_mask, candidate_tree_to_mask

__all__ = ["build_tree_mask", "candidate_tree_to_mask", "tree_attention", "tree_attention_plan", "tree_attention_cuda",
           "tree_attention_triton", "fused_tree_verify"]
