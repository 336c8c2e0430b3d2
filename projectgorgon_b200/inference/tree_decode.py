"""Tree verification inside a Hugging Face decoder step.

The reference's loop verifies a draft tree by running the backbone over
``[last_token, draft...]`` with plain causal attention and sequential
positions (``src/gorgon/inference/gorgon_loop.py:304-320``), then trims the
cache to the accepted path (``gorgon_loop.py:223-251``, ``:569-570``).  This
module runs that step with the operators' own contract
(``src/gorgon/kernels/tree_attention_ref.py:8-18`` on
``[ones(n, P) | build_tree_mask(parents)]``):

* every attention layer calls this package's tree attention, registered with
  transformers as the attention implementation ``"gorgon_tree"`` and switched
  on only for the verify forward: a step row sees the cached prefix and its
  own ancestors, nothing else (no dense mask is built);
* position ids are the prefix length plus the node's depth;
* ``verify_tree`` picks the accepted path on the device;
* the all-layer KV trim moves the accepted rows behind the prefix inside the
  model's own ``DynamicCache`` tensors, and the cache is cropped after them.

Prefill and plain decoding keep the model's configured attention; calling
``"gorgon_tree"`` without a tree raises.
"""
from __future__ import annotations

import contextlib
from dataclasses import dataclass
from typing import Iterator, List, Optional, Sequence, Tuple, Union

import torch

from ..kernels.tree_attention import tree_attention
from ..kernels.tree_mask import build_tree_mask
from .kv_cache import GorgonKVCache
from .verify import TreeVerifyResult, verify_tree

ATTN_IMPLEMENTATION = "gorgon_tree"
_registered = False


def gorgon_tree_attention(module, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                          attention_mask: Optional[torch.Tensor], scaling: Optional[float] = None,
                          dropout: float = 0.0, **kwargs) -> Tuple[torch.Tensor, None]:
    """Attention function in transformers' interface: ``query [B, Hq, n, D]``
    for the step's rows, ``key``/``value`` ``[B, Hkv, P + n, D]`` (the cache
    with the step's rows last).  The tree comes in the forward's keyword
    arguments: ``gorgon_parents`` ``[n]`` or ``[B, n]`` (-1 for a root), with
    optional ``gorgon_max_depth`` and ``gorgon_backend``.  Returns the output
    as ``[B, n, Hq, D]`` and no weights."""
    parents = kwargs.get("gorgon_parents")
    if parents is None:
        raise RuntimeError("the gorgon_tree attention runs tree verification only: pass gorgon_parents "
                           "(tree_forward does), and use the model's own attention for prefill")
    if dropout:
        raise RuntimeError("tree attention has no dropout (run the model in eval mode)")
    if attention_mask is not None:
        raise RuntimeError("tree attention takes its mask from gorgon_parents, not an attention mask")
    out = tree_attention(query, key, value, parents=parents, max_depth=kwargs.get("gorgon_max_depth"),
                         scale=scaling, backend=kwargs.get("gorgon_backend", "auto"))
    return out.transpose(1, 2), None


def register_tree_attention() -> str:
    """Registers ``gorgon_tree_attention`` with transformers (once) and
    returns its implementation name."""
    global _registered
    if not _registered:
        from transformers import AttentionInterface
        AttentionInterface.register(ATTN_IMPLEMENTATION, gorgon_tree_attention)
        _registered = True
    return ATTN_IMPLEMENTATION


@contextlib.contextmanager
def tree_attention_enabled(model) -> Iterator[None]:
    """Switches ``model`` to the tree attention for the block and restores
    its configured implementation afterwards, also on error."""
    name = register_tree_attention()
    cfg = model.config
    saved = cfg._attn_implementation
    cfg._attn_implementation = name
    try:
        yield
    finally:
        cfg._attn_implementation = saved


def tree_depths(parents: torch.Tensor) -> torch.Tensor:
    """Depth of every node (roots 0) of ``[n]`` or ``[B, n]`` parent arrays,
    on the parents' device, from the ancestor mask (ancestors per row - 1)."""
    return build_tree_mask(parents).sum(-1) - 1


def step_parents(parents: torch.Tensor) -> torch.Tensor:
    """Parents of the verify forward's rows ``[last_token, draft...]``: the
    last accepted token is row 0 and the single root, draft node ``t`` is row
    ``t + 1`` and hangs under row ``parents[t] + 1``, or under row 0 when it
    is a draft root."""
    par = parents if parents.dim() == 2 else parents.unsqueeze(0)
    shifted = torch.where(par >= 0, par + 1, torch.zeros_like(par))
    head = torch.full((par.shape[0], 1), -1, dtype=par.dtype, device=par.device)
    out = torch.cat([head, shifted], dim=1)
    return out if parents.dim() == 2 else out[0]


def _parents_on(parents: Union[Sequence[int], torch.Tensor], dev: torch.device) -> torch.Tensor:
    if isinstance(parents, torch.Tensor):
        return parents.to(device=dev, dtype=torch.int32)
    return torch.tensor(list(parents), dtype=torch.int32, device=dev)


def tree_forward(model, input_ids: torch.Tensor, parents: Union[Sequence[int], torch.Tensor], past_key_values,
                 max_depth: Optional[int] = None, backend: str = "auto"):
    """One forward of ``model`` over a tree of rows behind its cache.

    ``input_ids [B, n]`` are the rows' tokens, ``parents`` ``[n]`` or
    ``[B, n]`` their tree (-1: a root, which sees the prefix only).  Row ``i``
    gets position ``P + depth(i)`` (``P`` the cached length) and attends to
    the prefix and its own ancestors.  The rows' K/V are appended to
    ``past_key_values`` like any forward.  Returns the model's output
    (``.logits [B, n, V]``)."""
    dev = input_ids.device
    par = _parents_on(parents, dev)
    B, n = input_ids.shape
    if par.shape[-1] != n or (par.dim() == 2 and par.shape[0] != B):
        raise RuntimeError(f"parents {tuple(par.shape)} do not match input_ids {tuple(input_ids.shape)}")
    P = past_key_values.get_seq_length() if past_key_values is not None else 0
    depth = tree_depths(par)
    pos = (P + depth).to(torch.long)
    pos = pos.expand(B, n) if pos.dim() == 1 else pos
    with tree_attention_enabled(model):
        return model(input_ids=input_ids, position_ids=pos, past_key_values=past_key_values, use_cache=True,
                     gorgon_parents=par, gorgon_max_depth=max_depth, gorgon_backend=backend)


def hf_cache_layers(cache) -> Tuple[Tuple[torch.Tensor, torch.Tensor], ...]:
    """The per-layer ``(K, V)`` tensors ``[B, H, S, D]`` of a transformers
    ``DynamicCache`` (its ``layers[i].keys / .values``) or of a tuple of
    pairs, as the all-layer trim takes them."""
    layers = getattr(cache, "layers", None)
    if layers is not None:
        return tuple((l.keys, l.values) for l in layers)
    return tuple((k, v) for k, v in cache)


def trim_hf_cache(cache, src_idx: torch.Tensor, lens: torch.Tensor,
                  dst_start: Union[torch.Tensor, int, None] = None) -> None:
    """All-layer trim-on-reject in place on a transformers cache: for every
    layer, batch row ``b`` and head, row ``dst_start[b] + r`` takes row
    ``src_idx[b, r]`` for ``r < lens[b]`` (``GorgonKVCache.trim``)."""
    kv = GorgonKVCache()
    kv.update(hf_cache_layers(cache))
    kv.trim(src_idx, lens, dst_start)


@dataclass
class TreeStepResult:
    """One verify step.

    logits [B, n + 1, V]  rows: the last accepted token, then the draft nodes
    verify                the verifier's device outputs (``TreeVerifyResult``)
    accepted              host list of the accepted draft tokens (batch row 0)
    bonus                 the token that follows them
    seq_len               cache length after the trim
    """
    logits: torch.Tensor
    verify: TreeVerifyResult
    accepted: List[int]
    bonus: int
    seq_len: int


def tree_verify_step(model, cache, last_token: Union[int, torch.Tensor], draft: torch.Tensor,
                     parents: Union[Sequence[int], torch.Tensor], max_depth: Optional[int] = None,
                     backend: str = "auto") -> TreeStepResult:
    """Verifies a draft tree against ``model`` and leaves ``cache`` holding the
    prefix, the last token and the accepted path, as the reference's loop
    intends (``gorgon_loop.py:297-392``, ``:569-570``), for one sequence.

    ``last_token`` is the last accepted token (not yet in the cache),
    ``draft [n]`` or ``[1, n]`` the tree's tokens and ``parents`` its parent
    array.  Runs one tree forward over ``[last_token, draft...]``, the verifier
    with ``prompt_len = 1``, the all-layer trim of the accepted rows to just
    after the last token, and crops the cache there."""
    dev = draft.device
    dr = draft if draft.dim() == 2 else draft.unsqueeze(0)
    if dr.shape[0] != 1:
        raise RuntimeError("tree_verify_step verifies one sequence (a transformers cache has one length "
                           "for every batch row)")
    n = dr.shape[1]
    par = _parents_on(parents, dev).reshape(-1)
    if par.numel() != n:
        raise RuntimeError(f"parents has {par.numel()} entries for {n} draft nodes")
    last = torch.as_tensor(last_token, device=dev).reshape(1, 1).to(dr.dtype)
    P = cache.get_seq_length()
    ids = torch.cat([last, dr], dim=1).to(torch.long)
    out = tree_forward(model, ids, step_parents(par), cache, max_depth=None if max_depth is None else max_depth + 1,
                       backend=backend)
    res = verify_tree(out.logits[0], dr[0], par, prompt_len=1)
    # accepted node path[i] sits at row P + 1 + path[i]; it moves to P + 1 + i
    src = (P + 1 + res.path.clamp(min=0)).reshape(1, n)
    trim_hf_cache(cache, src, res.accepted_len.reshape(1), P + 1)
    acc_len = int(res.accepted_len.item())
    cache.crop(P + 1 + acc_len)
    path = res.path[:acc_len].tolist()
    toks = dr[0].tolist()
    return TreeStepResult(logits=out.logits, verify=res, accepted=[toks[i] for i in path],
                          bonus=int(res.bonus.item()), seq_len=P + 1 + acc_len)
