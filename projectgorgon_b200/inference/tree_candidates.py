"""Candidate-tree builder on the GPU.

``build_candidate_tree`` keeps the reference's signature and result type
(``src/gorgon/inference/tree_candidates.py:92-245``): it runs the Medusa heads
on the hidden state, then hands their logits to ``gorgon_candidate_tree``,
which computes every head's top-k, the softmax over it and the entropy of the
full distribution (``_topk_per_head``, ``:42-81``) and assembles the tree on
the device, with the reference's budget (``max_candidates``), confidence
threshold, path-confidence and entropy-weighting rules.  The reference
synchronises with the host once per head and loops over the nodes in Python;
here the only synchronisation is the one the result type needs (``parents``
is a Python list).

``build_candidate_trees`` is the batched form for a decode loop: logits of
``B`` sequences in, device tensors out, no synchronisation at all.
``head_candidate_trees`` takes the heads' ``lm_head`` inputs and weights
instead of logits: the Linear runs inside the statistics kernel
(``MedusaHead.forward``'s last layer fused with ``_topk_per_head``).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import List, NamedTuple, Optional, Sequence

import torch

from .. import _abi
from .._util import gorgon_dtype, on_device, require_cuda, stream_ptr, workspace

__all__ = ["CandidateTree", "CandidateTrees", "HeadStatistics", "build_candidate_tree", "build_candidate_trees",
           "head_candidate_trees", "head_statistics", "max_tree_nodes", "medusa_head_inputs"]


@dataclass
class CandidateTree:
    """Flat candidate tree, as the reference's ``CandidateTree``
    (``tree_candidates.py:17-30``): tokens (int64, device), parents (list,
    -1 = root), depth, scores (each node's probability, float32, device)."""
    tokens: torch.Tensor
    parents: List[int]
    depth: int
    scores: Optional[torch.Tensor] = None


class CandidateTrees(NamedTuple):
    """Trees of a batch, on the device.  Row ``b`` holds ``n_nodes[b]`` nodes;
    the slots after them hold token -1, parent -1, probability 0."""
    tokens: torch.Tensor    # int64 [B, max_nodes]
    parents: torch.Tensor   # int32 [B, max_nodes], -1 = root
    scores: torch.Tensor    # float32 [B, max_nodes]
    n_nodes: torch.Tensor   # int32 [B]
    depth: int


class HeadStatistics(NamedTuple):
    """Per (sequence, head): the top-k logits and ids (descending, equal logits
    by ascending id), the softmax over them and the full distribution's entropy."""
    ids: torch.Tensor       # int32 [B, L, k]
    scores: torch.Tensor    # float32 [B, L, k]
    probs: torch.Tensor     # float32 [B, L, k]
    entropy: torch.Tensor   # float32 [B, L]


def max_tree_nodes(top_k: int, depth: int, vocab: Optional[int] = None,
                   max_candidates: Optional[int] = None) -> int:
    """Largest tree the rules allow: ``k + k^2 + ... + k^depth`` with
    ``k = min(top_k, vocab)``, capped by the budget."""
    k = top_k if vocab is None else min(top_k, vocab)
    total, width = 0, 1
    for _ in range(depth):
        width *= k
        total += width
        if max_candidates is not None and total >= max_candidates:
            return max(int(max_candidates), 0)
    return total if max_candidates is None else min(total, max(int(max_candidates), 0))


def _logits3(logits: torch.Tensor) -> torch.Tensor:
    require_cuda("logits", logits)
    if logits.dim() == 2:
        logits = logits.unsqueeze(0)
    if logits.dim() != 3:
        raise RuntimeError(f"logits must be [levels, vocab] or [batch, levels, vocab], got {tuple(logits.shape)}")
    if logits.dtype not in (torch.float32, torch.bfloat16, torch.float16):
        raise RuntimeError(f"logits dtype {logits.dtype} is not float32 / bfloat16 / float16")
    if logits.stride(-1) != 1:
        logits = logits.contiguous()
    return logits


def _tree_params(dtype: torch.dtype, B: int, L: int, V: int, dev: torch.device, top_k: int,
                 max_candidates: Optional[int], confidence_threshold: float, use_path_confidence: bool,
                 entropy_weighted: bool, max_nodes: int, stats: Optional[HeadStatistics]):
    """The tree part of a parameter block (rules, outputs, statistics) and the
    trees it will fill."""
    cap = max(int(max_nodes), 1)
    out = CandidateTrees(tokens=torch.empty(B, cap, dtype=torch.int64, device=dev),
                         parents=torch.empty(B, cap, dtype=torch.int32, device=dev),
                         scores=torch.empty(B, cap, dtype=torch.float32, device=dev),
                         n_nodes=torch.empty(B, dtype=torch.int32, device=dev), depth=L)
    p = _abi.CandidateTreeParams()
    p.dtype = gorgon_dtype(dtype)
    p.batch, p.levels, p.vocab = B, L, V
    p.top_k = int(top_k)
    p.max_candidates = -1 if max_candidates is None else int(max_candidates)
    p.confidence_threshold = float(confidence_threshold)
    p.use_path_confidence, p.entropy_weighted = int(bool(use_path_confidence)), int(bool(entropy_weighted))
    p.max_nodes = cap
    p.tokens, p.parents, p.probs, p.n_nodes = (out.tokens.data_ptr(), out.parents.data_ptr(),
                                               out.scores.data_ptr(), out.n_nodes.data_ptr())
    if stats is not None:
        p.topk_ids, p.topk_scores = stats.ids.data_ptr(), stats.scores.data_ptr()
        p.topk_probs, p.entropy = stats.probs.data_ptr(), stats.entropy.data_ptr()
    return p, out


def _run(lg: torch.Tensor, top_k: int, max_candidates: Optional[int], confidence_threshold: float,
         use_path_confidence: bool, entropy_weighted: bool, max_nodes: int, stats: Optional[HeadStatistics]):
    B, L, V = lg.shape
    dev = lg.device
    p, out = _tree_params(lg.dtype, B, L, V, dev, top_k, max_candidates, confidence_threshold,
                          use_path_confidence, entropy_weighted, max_nodes, stats)
    p.logits, p.logits_stride_b, p.logits_stride_l = lg.data_ptr(), lg.stride(0), lg.stride(1)
    lib = _abi.lib()
    with on_device(dev):
        nbytes = lib.gorgon_candidate_tree_workspace_size(p)
        ws = workspace(nbytes, dev)
        _abi.check(lib.gorgon_candidate_tree(p, ws.data_ptr(), ws.numel(), stream_ptr(dev)),
                   "gorgon_candidate_tree")
    return out


def build_candidate_trees(logits: torch.Tensor, top_k: int = 4, max_candidates: Optional[int] = None,
                          confidence_threshold: float = 0.0, use_path_confidence: bool = False,
                          entropy_weighted: bool = False, max_nodes: Optional[int] = None) -> CandidateTrees:
    """Candidate trees of a batch from its heads' logits ``[B, L, V]`` (or one
    sequence's ``[L, V]``), level ``l + 1`` from head ``l``.  The rules are
    ``build_candidate_tree``'s; ``max_nodes`` (default: the largest tree the
    rules allow) is the capacity per row, at most 4096 -- a tree cut there
    sets device error bit 5."""
    lg = _logits3(logits)
    B, L, V = lg.shape
    cap = max_nodes if max_nodes is not None else max_tree_nodes(top_k, L, V, max_candidates)
    return _run(lg, top_k, max_candidates, confidence_threshold, use_path_confidence, entropy_weighted,
                cap, None)


def head_statistics(logits: torch.Tensor, top_k: int) -> HeadStatistics:
    """The per-head part alone (``_topk_per_head``, ``tree_candidates.py:42-81``)
    for logits ``[B, L, V]`` or ``[L, V]``; entries past ``min(top_k, V)`` are
    -1 / -inf / 0."""
    lg = _logits3(logits)
    B, L, V = lg.shape
    dev = lg.device
    st = HeadStatistics(ids=torch.empty(B, L, top_k, dtype=torch.int32, device=dev),
                        scores=torch.empty(B, L, top_k, dtype=torch.float32, device=dev),
                        probs=torch.empty(B, L, top_k, dtype=torch.float32, device=dev),
                        entropy=torch.empty(B, L, dtype=torch.float32, device=dev))
    _run(lg, top_k, 0, 0.0, False, False, 1, st)
    if logits.dim() == 2:
        st = HeadStatistics(*(t[0] for t in st))
    return st


MAX_FUSED_BATCH = 4


def head_candidate_trees(hidden: torch.Tensor, lm_heads: Sequence[torch.Tensor], top_k: int = 4,
                         max_candidates: Optional[int] = None, confidence_threshold: float = 0.0,
                         use_path_confidence: bool = False, entropy_weighted: bool = False,
                         max_nodes: Optional[int] = None, logits_dtype: Optional[torch.dtype] = None,
                         return_statistics: bool = False):
    """Candidate trees straight from the heads' last Linear, with the logits
    never stored (``gorgon_head_candidate_tree``).

    ``hidden [B, L, H]`` (or ``[L, H]``) is the input of head ``l``'s
    ``lm_head`` for sequence ``b`` (after the head's norm and residual blocks:
    ``medusa_head_inputs``); ``lm_heads`` are the ``L`` weights ``[V, H]``
    (``nn.Linear.weight``), bf16 or f16 like ``hidden``.  Every logit
    ``hidden[b, l] . lm_heads[l][v]`` is accumulated in fp32 and rounded to
    ``logits_dtype`` (default: the weights' dtype, what the Linear returns);
    the rules and results are ``build_candidate_trees``'.  ``B <= 4``.  With
    ``return_statistics`` also the ``HeadStatistics``."""
    require_cuda("hidden", hidden)
    x = hidden if hidden.dim() == 3 else hidden.unsqueeze(0)
    if x.dim() != 3:
        raise RuntimeError(f"hidden must be [levels, hidden] or [batch, levels, hidden], got {tuple(hidden.shape)}")
    B, L, H = x.shape
    if len(lm_heads) != L:
        raise RuntimeError(f"{len(lm_heads)} lm_head weights for {L} levels")
    if B > MAX_FUSED_BATCH:
        raise RuntimeError(f"the fused heads take at most {MAX_FUSED_BATCH} sequences (got {B}); "
                           "run the heads and use build_candidate_trees")
    dev = x.device
    for w in lm_heads:
        require_cuda("lm_head weights", w)
        if w.dim() != 2 or w.shape[1] != H or w.shape[0] != lm_heads[0].shape[0]:
            raise RuntimeError(f"lm_head weights must all be [vocab, {H}], got {tuple(w.shape)}")
        if w.dtype != x.dtype or w.device != dev:
            raise RuntimeError("lm_head weights and hidden must share dtype and device")
    # one row stride for every level, hidden contiguous (Linear weights already are)
    ws_list = list(lm_heads)
    if any(w.stride(1) != 1 or w.stride(0) != ws_list[0].stride(0) for w in ws_list):
        ws_list = [w.contiguous() for w in ws_list]
    if x.stride(-1) != 1:
        x = x.contiguous()
    V = ws_list[0].shape[0]
    out_dt = logits_dtype if logits_dtype is not None else x.dtype
    cap = max_nodes if max_nodes is not None else max_tree_nodes(top_k, L, V, max_candidates)
    stats = None
    if return_statistics:
        stats = HeadStatistics(ids=torch.empty(B, L, top_k, dtype=torch.int32, device=dev),
                               scores=torch.empty(B, L, top_k, dtype=torch.float32, device=dev),
                               probs=torch.empty(B, L, top_k, dtype=torch.float32, device=dev),
                               entropy=torch.empty(B, L, dtype=torch.float32, device=dev))
    tp, out = _tree_params(out_dt, B, L, V, dev, top_k, max_candidates, confidence_threshold,
                           use_path_confidence, entropy_weighted, cap, stats)
    p = _abi.HeadCandidateParams()
    p.tree = tp
    p.x_dtype = gorgon_dtype(x.dtype)
    p.hidden, p.hidden_stride_b, p.hidden_stride_l = x.data_ptr(), x.stride(0), x.stride(1)
    p.hidden_size = H
    ptrs = _abi.pointer_array([w.data_ptr() for w in ws_list])
    p.lm_head = ctypes.cast(ptrs, ctypes.c_void_p)
    p.lm_head_stride_v = ws_list[0].stride(0)
    lib = _abi.lib()
    with on_device(dev):
        nbytes = lib.gorgon_head_candidate_tree_workspace_size(p)
        ws = workspace(nbytes, dev)
        _abi.check(lib.gorgon_head_candidate_tree(p, ws.data_ptr(), ws.numel(), stream_ptr(dev)),
                   "gorgon_head_candidate_tree")
    return (out, stats) if return_statistics else out


def medusa_head_inputs(heads, hidden: torch.Tensor) -> torch.Tensor:
    """The input of every head's ``lm_head``: ``hidden`` (``[..., H]``, one
    row per sequence) through the head's ``norm`` and residual ``blocks``
    (``MedusaHead.forward`` without its last Linear,
    ``src/gorgon/models/medusa_heads.py:42-47``), as ``[B, L, H]``."""
    x0 = hidden.reshape(-1, hidden.shape[-1])
    rows = []
    with torch.no_grad():
        for head in heads:
            x = x0
            norm = getattr(head, "norm", None)
            if norm is not None:
                x = norm(x)
            for block in getattr(head, "blocks", ()):
                x = block(x)
            rows.append(x)
    return torch.stack(rows, dim=1)


def build_candidate_tree(heads, hidden: torch.Tensor, top_k: int = 4, max_depth: Optional[int] = None,
                         max_candidates: Optional[int] = None, confidence_threshold: float = 0.0,
                         use_path_confidence: bool = False, entropy_weighted: bool = False,
                         fused: bool = False) -> CandidateTree:
    """Drop-in for the reference's ``build_candidate_tree``
    (``tree_candidates.py:92-245``): runs ``heads[:depth]`` on ``hidden``
    (``depth = min(max_depth or len(heads), len(heads))``), then builds the
    tree on the device.  ``hidden`` must be a CUDA tensor.  With ``fused``
    (heads with a bias-free ``lm_head`` Linear, bf16/f16) the heads' last
    Linear runs inside the statistics kernel (``head_candidate_trees``)."""
    require_cuda("hidden", hidden)
    num_heads = len(heads)
    depth = min(max_depth or num_heads, num_heads)
    if fused:
        for head in heads[:depth]:
            if getattr(head, "lm_head", None) is None or head.lm_head.bias is not None:
                raise RuntimeError("fused=True needs heads whose lm_head is a Linear without bias")
        x = medusa_head_inputs(heads[:depth], hidden.reshape(-1, hidden.shape[-1])[:1])
        trees = head_candidate_trees(x, [h.lm_head.weight for h in heads[:depth]], top_k=top_k,
                                     max_candidates=max_candidates, confidence_threshold=confidence_threshold,
                                     use_path_confidence=use_path_confidence, entropy_weighted=entropy_weighted)
        n = int(trees.n_nodes[0].item())
        return CandidateTree(tokens=trees.tokens[0, :n], parents=trees.parents[0, :n].tolist(), depth=depth,
                             scores=trees.scores[0, :n])
    rows = []
    with torch.no_grad():
        for head in heads[:depth]:
            lg = head(hidden)
            if lg.dim() == 3:
                lg = lg[0, 0]
            elif lg.dim() == 2:
                lg = lg[0]
            rows.append(lg)
    logits = torch.stack(rows)
    trees = build_candidate_trees(logits, top_k=top_k, max_candidates=max_candidates,
                                  confidence_threshold=confidence_threshold,
                                  use_path_confidence=use_path_confidence, entropy_weighted=entropy_weighted)
    n = int(trees.n_nodes[0].item())
    return CandidateTree(tokens=trees.tokens[0, :n], parents=trees.parents[0, :n].tolist(), depth=depth,
                         scores=trees.scores[0, :n])
