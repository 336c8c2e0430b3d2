"""``fused_tree_verify`` (``src/gorgon/kernels/fused_tree_verify_triton.py:110-172``).

Mask-free tree attention: the kernel walks ``parents`` up ``max_depth`` hops
per row instead of reading a mask.  Ancestors farther than ``max_depth`` hops
are not visible, as in the reference.  ``k``/``v`` may carry a prefix (rows
before the tree), and the batched / grouped-query forms of ``tree_attention``
are accepted.
"""
from __future__ import annotations

from typing import List, Union

import torch

from .tree_attention import tree_attention


def fused_tree_verify(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                      parents: Union[List[int], torch.Tensor], max_depth: int = 5,
                      **kwargs) -> torch.Tensor:
    if not q.is_cuda or not k.is_cuda or not v.is_cuda:
        raise ValueError("q, k, v must be CUDA tensors.")
    return tree_attention(q, k, v, parents=parents, max_depth=max_depth, **kwargs)
