"""``tree_attention_cuda`` (``src/gorgon/kernels/tree_attention_cuda.py:24-38``).

The reference JIT-builds an fp32 SIMT kernel and returns float32; this name
now runs the sm_100a library and likewise returns float32.
"""
from __future__ import annotations

import torch

from .tree_attention import tree_attention


def tree_attention_cuda(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                        mask: torch.Tensor) -> torch.Tensor:
    if not (q.is_cuda and k.is_cuda and v.is_cuda and mask.is_cuda):
        raise ValueError("q, k, v, mask must be CUDA tensors")
    return tree_attention(q, k, v, mask, out_dtype=torch.float32)
