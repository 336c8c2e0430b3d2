"""Tree verifier on the GPU: argmax, draft match and longest accepted path.

``verify_tree`` is the tensor-level form of the vectorised verifier inside
``_verify_tree_candidates`` (``src/gorgon/inference/gorgon_loop.py:328-392``):
one launch computes every needed row's argmax, matches drafts and picks the
winning path, and its outputs stay on the device (no ``.cpu()`` sync).
``accept_draft_tokens`` keeps the reference's chain API
(``gorgon_loop.py:161-184``) and returns Python lists like the original.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Sequence, Tuple, Union

import torch

from .. import _abi
from .._util import gorgon_dtype, on_device, require_cuda, stream_ptr, workspace


@dataclass
class TreeVerifyResult:
    """Device tensors (int32) of one verification.

    accepted_len [B]   number of accepted draft tokens on the winning path
    path [B, n]        winning node indices from the root, -1 padded
    bonus [B]          argmax after the last accepted node (or after the prompt)
    best_node [B]      last accepted node, -1 when nothing was accepted
    hidden_row [B]     logits row whose hidden state continues decoding
    pred [B, n + 1]    argmax of rows prompt_len - 1 .. prompt_len - 1 + n
    """
    accepted_len: torch.Tensor
    path: torch.Tensor
    bonus: torch.Tensor
    best_node: torch.Tensor
    hidden_row: torch.Tensor
    pred: torch.Tensor

    def accepted_tokens(self, draft: torch.Tensor) -> List[List[int]]:
        """Host lists of accepted token ids per batch row (synchronises)."""
        d = draft if draft.dim() == 2 else draft.unsqueeze(0)
        lens = self.accepted_len.reshape(-1).tolist()
        paths = self.path.reshape(len(lens), -1).tolist()
        dl = d.tolist()
        return [[dl[b][paths[b][i]] for i in range(lens[b])] for b in range(len(lens))]


def verify_tree(logits: torch.Tensor, draft: torch.Tensor,
                parents: Union[Sequence[int], torch.Tensor], prompt_len: int = 1) -> TreeVerifyResult:
    """Verify candidate trees against verifier logits.

    logits  [R, V] or [B, R, V] (float32 / bfloat16 / float16, CUDA)
    draft   [n] or [B, n] token ids of the tree nodes
    parents [n] or [B, n] (list or tensor), -1 marks a root

    Node ``t`` is checked against ``argmax(logits[prompt_len - 1])`` when it is
    a root and ``argmax(logits[prompt_len + parents[t]])`` otherwise; the first
    root-to-leaf path in DFS order with the longest accepted prefix wins
    (``gorgon_loop.py:342-371``).  With a KV cache the reference uses
    ``prompt_len = 1`` (``gorgon_loop.py:297-300``).
    """
    require_cuda("logits and draft", logits, draft)
    dev = logits.device
    lg = logits if logits.dim() == 3 else logits.unsqueeze(0)
    if lg.stride(-1) != 1:
        lg = lg.contiguous()
    B, R, V = lg.shape
    dr = draft if draft.dim() == 2 else draft.unsqueeze(0)
    dr = dr.to(device=dev, dtype=torch.int32).contiguous()
    if dr.shape[0] != B:
        raise RuntimeError(f"draft batch {dr.shape[0]} != logits batch {B}")
    n = dr.shape[1]
    if isinstance(parents, torch.Tensor):
        par = parents.to(device=dev, dtype=torch.int32).contiguous()
    else:
        par = torch.tensor(list(parents), dtype=torch.int32, device=dev)
    if par.dim() == 1:
        if par.numel() != n:
            raise RuntimeError(f"parents has {par.numel()} entries for {n} draft nodes")
        psb = 0
    elif par.shape == (B, n):
        psb = par.stride(0)
    else:
        raise RuntimeError(f"parents must be [n] or [B, n], got {tuple(par.shape)}")
    i32 = dict(dtype=torch.int32, device=dev)
    res = TreeVerifyResult(
        accepted_len=torch.empty(B, **i32), path=torch.empty(B, n, **i32),
        bonus=torch.empty(B, **i32), best_node=torch.empty(B, **i32),
        hidden_row=torch.empty(B, **i32), pred=torch.empty(B, n + 1, **i32))
    p = _abi.VerifyParams()
    p.dtype = gorgon_dtype(lg.dtype)
    p.logits, p.logits_stride_b, p.logits_stride_r = lg.data_ptr(), lg.stride(0), lg.stride(1)
    p.batch, p.rows, p.vocab, p.n, p.prompt_len = B, R, V, n, int(prompt_len)
    p.draft, p.draft_stride_b = dr.data_ptr(), dr.stride(0)
    p.parents, p.parents_stride_b = par.data_ptr(), psb
    p.pred, p.accepted_len, p.path = res.pred.data_ptr(), res.accepted_len.data_ptr(), res.path.data_ptr()
    p.bonus, p.best_node, p.hidden_row = res.bonus.data_ptr(), res.best_node.data_ptr(), res.hidden_row.data_ptr()
    lib = _abi.lib()
    with on_device(dev):
        nbytes = lib.gorgon_verify_workspace_size(p)
        ws = workspace(nbytes, dev)
        _abi.check(lib.gorgon_verify(p, ws.data_ptr(), ws.numel(), stream_ptr(dev)), "gorgon_verify")
    if logits.dim() == 2:
        res = TreeVerifyResult(*(t[0] for t in (res.accepted_len, res.path, res.bonus, res.best_node,
                                               res.hidden_row, res.pred)))
    return res


def accept_draft_tokens(draft: List[int], logits: torch.Tensor) -> Tuple[List[int], int]:
    """Greedy chain acceptance: accept consecutive draft tokens that match the
    verifier's argmax, stop at the first mismatch.  Returns the accepted tokens
    and the rejected index (``len(draft)`` when all match)."""
    require_cuda("logits", logits)
    n = len(draft)
    if n == 0:
        return [], 0
    dev = logits.device
    d = torch.tensor(list(draft), dtype=torch.int32, device=dev)
    chain = list(range(-1, n - 1))
    res = verify_tree(logits[:n], d, chain, prompt_len=1)
    acc = int(res.accepted_len.item())
    return [int(t) for t in draft[:acc]], (acc if acc < n else n)
