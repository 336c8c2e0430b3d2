"""``tree_attention_triton`` (``src/gorgon/kernels/tree_attention_triton.py:86-127``).

Kept as a name only: it runs the sm_100a CUDA library (no Triton) and returns
``q``'s dtype like the original's ``torch.empty_like(q)``.
"""
from __future__ import annotations

import torch

from .tree_attention import tree_attention


def tree_attention_triton(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                          mask: torch.Tensor) -> torch.Tensor:
    if not q.is_cuda or not k.is_cuda or not v.is_cuda or not mask.is_cuda:
        raise ValueError("q, k, v, and mask must be CUDA tensors.")
    return tree_attention(q, k, v, mask)
