"""``build_tree_mask`` on the GPU (``src/gorgon/kernels/tree_mask.py:16-44``)."""
from __future__ import annotations

from typing import Optional, Sequence, Union

import torch

from .. import _abi
from .._util import on_device, parents_tensor, stream_ptr


def build_tree_mask(parents: Union[Sequence[int], torch.Tensor], depth: Optional[int] = None,
                    *, device: Union[torch.device, str, None] = None) -> torch.Tensor:
    """Boolean ancestor mask: ``mask[i, j]`` is true iff ``j == i`` or ``j`` is
    within ``depth`` parent hops above ``i`` (``depth=None``: ``len(parents)``
    hops, the reference's default).  ``parents`` is a list, or an int tensor
    ``[N]`` / ``[B, N]`` (one mask per row).  The mask is built on a CUDA device:
    ``device``, the tensor's own device, or the current one."""
    if isinstance(parents, torch.Tensor) and parents.is_cuda:
        dev = parents.device
    else:
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    if dev.type != "cuda":
        raise ValueError("build_tree_mask runs on a CUDA device.")
    par = parents_tensor(parents, dev)
    batched = par.dim() == 2
    if par.dim() not in (1, 2):
        raise RuntimeError("parents must be [N] or [B, N]")
    p2 = par if batched else par.unsqueeze(0)
    B, n = p2.shape
    out = torch.empty((B, n, n), dtype=torch.bool, device=dev)
    d = -1 if depth is None else int(depth)
    with on_device(dev):
        _abi.check(_abi.lib().gorgon_tree_mask(p2.data_ptr(), B, n, p2.stride(0), d, out.data_ptr(),
                                               stream_ptr(dev)), "gorgon_tree_mask")
    return out if batched else out[0]


def candidate_tree_to_mask(tree) -> torch.Tensor:
    """Mask of a candidate tree with ``tree.depth`` hops
    (``src/gorgon/inference/tree_candidates.py:248-279``)."""
    dev = tree.tokens.device if getattr(tree, "tokens", None) is not None and tree.tokens.is_cuda else None
    return build_tree_mask(tree.parents, tree.depth, device=dev)
