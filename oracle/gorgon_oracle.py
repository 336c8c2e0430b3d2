"""CPU oracle for the tree-verification path (test infrastructure only).

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs
of ``bench.py`` may import it.  The CUDA library in ``projectgorgon_b200`` never
calls into it and has no CPU fallback.

Every function restates one piece of ProjectGorgon's reference code in numpy
(pure-Python loops only where the reference itself loops over a small tree).
Each docstring names the reference file:line it follows.  Parity is pinned by
``tests/golden/*.npz``: vectors produced by running the reference's own
functions (``tests/golden/make_golden.py``), which ``tests/test_oracle.py``
checks this module against.

Conventions shared with the CUDA path:

* ``parents[i]`` is the parent of tree node ``i``; ``-1`` marks a root.
* A tree of ``n`` nodes is appended after a prefix of ``P`` key/value rows, so a
  sequence has ``L = P + n`` rows and tree node ``i`` lives in row ``P + i``.
* Grouped-query attention: query head ``h`` reads kv head ``h // (Hq // Hkv)``.
"""
from __future__ import annotations

import math
from typing import List, Optional, Sequence, Tuple

import numpy as np

__all__ = [
    "build_tree_mask",
    "prefix_tree_mask",
    "tree_attention",
    "fused_tree_verify",
    "tree_attention_batched",
    "accept_draft_tokens",
    "get_tree_paths",
    "verify_tree",
    "apply_cache_slice",
    "kv_trim",
    "head_topk",
    "build_candidate_tree",
]


# --------------------------------------------------------------------------
# A1: tree mask
# --------------------------------------------------------------------------
def build_tree_mask(parents: Sequence[int], depth: Optional[int] = None) -> np.ndarray:
    """Ancestor mask, ``mask[i, j]`` true iff j == i or j is within ``depth``
    parent hops above i.

    Follows ``src/gorgon/kernels/tree_mask.py:16-44``: start from the identity,
    then ``depth`` rounds (default ``len(parents)``) of vectorised pointer
    jumping, each marking the current ancestor and moving one hop up.  A
    negative parent ends a chain (``valid = current >= 0`` at :35).
    """
    par = np.asarray(list(parents), dtype=np.int64)
    n = par.shape[0]
    mask = np.eye(n, dtype=bool)
    max_iter = n if depth is None else int(depth)
    current = par.copy()
    rows_all = np.arange(n)
    for _ in range(max_iter):
        valid = current >= 0
        if not valid.any():
            break
        rows = rows_all[valid]
        cols = current[valid]
        mask[rows, cols] = True
        nxt = np.full_like(current, -1)
        nxt[valid] = par[current[valid]]
        current = nxt
    return mask


def prefix_tree_mask(parents: Sequence[int], prefix_len: int,
                     depth: Optional[int] = None) -> np.ndarray:
    """``[ones(n, P) | build_tree_mask(parents, depth)]``: the tree rows see the
    whole prefix plus their own ancestors.  This is how a prefix is expressed
    through the reference's rectangular-mask form of ``tree_attention_ref``
    (``src/gorgon/kernels/tree_attention_ref.py:8-18`` accepts ``[N, M]``)."""
    tm = build_tree_mask(parents, depth)
    n = tm.shape[0]
    return np.concatenate([np.ones((n, int(prefix_len)), dtype=bool), tm], axis=1)


# --------------------------------------------------------------------------
# A2 / A5: attention
# --------------------------------------------------------------------------
def tree_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, mask: np.ndarray,
                   dtype=np.float32) -> np.ndarray:
    """``softmax(q k^T / sqrt(d), masked -inf) v`` for one 2-D slice.

    Follows ``src/gorgon/kernels/tree_attention_ref.py:8-18``: scale is
    ``1/sqrt(q.shape[-1])``; masked scores are ``-inf`` before the softmax, so
    a row whose mask is all false becomes NaN exactly as ``torch.softmax``
    makes it.  ``dtype`` is the arithmetic type (float32 like the reference, or
    float64 for a tighter check).
    """
    q = np.asarray(q, dtype=dtype)
    k = np.asarray(k, dtype=dtype)
    v = np.asarray(v, dtype=dtype)
    mask = np.asarray(mask, dtype=bool)
    dim = q.shape[-1]
    scores = (q @ k.T) * dtype(1.0 / math.sqrt(dim))
    scores = np.where(mask, scores, dtype(-np.inf))
    with np.errstate(invalid="ignore", over="ignore"):
        mx = scores.max(axis=-1, keepdims=True)
        e = np.exp(scores - mx)
        w = e / e.sum(axis=-1, keepdims=True)
    return (w @ v).astype(dtype)


def fused_tree_verify(q, k, v, parents, max_depth: int = 5, dtype=np.float32):
    """Mask-free form: the mask is the ``max_depth``-hop ancestor walk.

    Follows ``src/gorgon/kernels/fused_tree_verify_triton.py:52-63`` (row i sees
    itself plus ``parents`` followed up to ``MAX_DEPTH`` hops), which equals
    ``build_tree_mask(parents, depth=max_depth)``; keys may carry a prefix of
    ``k.shape[0] - len(parents)`` fully visible rows.
    """
    n = len(parents)
    prefix = k.shape[0] - n
    mask = prefix_tree_mask(parents, prefix, max_depth)
    return tree_attention(q, k, v, mask, dtype=dtype)


def tree_attention_batched(q: np.ndarray, k: np.ndarray, v: np.ndarray, *,
                           parents=None, max_depth: Optional[int] = None,
                           mask: Optional[np.ndarray] = None,
                           kv_lens: Optional[Sequence[int]] = None,
                           dtype=np.float32) -> np.ndarray:
    """The batched / grouped-query extension, defined slice by slice.

    ``q[B, Hq, n, D]``, ``k, v[B, Hkv, L, D]`` (``L`` may exceed a sequence's
    own ``kv_lens[b]``; rows beyond it are ignored).  Each (b, h) slice is
    ``tree_attention(q[b,h], k[b,h//G,:L_b], v[b,h//G,:L_b], M_b)`` with
    ``M_b = [ones(n, L_b - n) | build_tree_mask(parents_b, max_depth)]`` when
    ``parents`` is given (``parents`` is ``[n]`` or ``[B, n]``), or ``mask``
    (``[n, L_b]`` full, or ``[n, n]`` tree-only with the prefix visible).
    The reference is 2-D only (``tree_attention_ref.py:14`` uses ``k.T``), so
    this per-slice loop is its only batched meaning.
    """
    B, Hq, n, D = q.shape
    Hkv = k.shape[1]
    G = Hq // Hkv
    out = np.zeros((B, Hq, n, D), dtype=dtype)
    for b in range(B):
        L = k.shape[2] if kv_lens is None else int(kv_lens[b])
        P = L - n
        if parents is not None:
            par = np.asarray(parents)
            pb = par[b] if par.ndim == 2 else par
            m = prefix_tree_mask(list(pb), P, max_depth)
        else:
            mm = np.asarray(mask, dtype=bool)
            mb = mm[b] if mm.ndim == 3 else mm
            if mb.shape[1] == L:
                m = mb
            else:
                m = np.concatenate([np.ones((n, P), dtype=bool), mb], axis=1)
        for h in range(Hq):
            out[b, h] = tree_attention(q[b, h], k[b, h // G, :L], v[b, h // G, :L], m, dtype=dtype)
    return out


# --------------------------------------------------------------------------
# V1 / V2: verifier
# --------------------------------------------------------------------------
def accept_draft_tokens(draft: Sequence[int], logits: np.ndarray) -> Tuple[List[int], int]:
    """Greedy chain acceptance, ``src/gorgon/inference/gorgon_loop.py:161-184``:
    accept ``draft[i]`` while ``argmax(logits[i]) == draft[i]``; return the
    accepted tokens and the first rejected index (``len(draft)`` if none)."""
    accepted: List[int] = []
    rejected_at = len(draft)
    for idx, tok in enumerate(draft):
        if int(np.argmax(logits[idx])) == int(tok):
            accepted.append(int(tok))
        else:
            rejected_at = idx
            break
    return accepted, rejected_at


def get_tree_paths(parents: Sequence[int]) -> List[List[int]]:
    """All root-to-leaf paths in DFS order (roots ascending, children in index
    order), ``src/gorgon/inference/tree_candidates.py:282-311``."""
    n = len(parents)
    children: List[List[int]] = [[] for _ in range(n)]
    roots: List[int] = []
    for i, p in enumerate(parents):
        if p == -1:
            roots.append(i)
        else:
            children[p].append(i)
    paths: List[List[int]] = []

    def dfs(node: int, path: List[int]) -> None:
        path.append(node)
        if not children[node]:
            paths.append(list(path))
        else:
            for c in children[node]:
                dfs(c, path)
        path.pop()

    for r in roots:
        dfs(r, [])
    return paths


def verify_tree(logits: np.ndarray, draft: Sequence[int], parents: Sequence[int],
                prompt_len: int = 1) -> dict:
    """Longest accepted root-to-leaf path and bonus token for one sequence.

    Restates the vectorised verifier of
    ``src/gorgon/inference/gorgon_loop.py:328-392`` on logits given directly
    (the original takes an HF model; ``tests/golden/make_golden.py`` runs the
    original with a fake model to pin this restatement):

    * ``pred = argmax(logits, -1)`` (first index on ties, NaN counts as max).
    * Along each path from :func:`get_tree_paths`, node t is accepted while
      ``draft[t] == pred[row]`` with ``row = prompt_len - 1`` for a root and
      ``prompt_len + parent`` otherwise (:345-358).
    * The first path with a strictly longer accepted prefix wins (:368-371).
    * The bonus is ``pred[prompt_len + last_accepted]``, or
      ``pred[prompt_len - 1]`` when nothing was accepted (:360-375); the same
      row is the hidden-state row (:377-383).
    """
    pred = np.argmax(np.asarray(logits, dtype=np.float64), axis=-1)
    paths = get_tree_paths(parents)
    best: List[int] = []
    best_path_nodes: List[int] = []
    best_bonus = -1
    for path in paths:
        acc: List[int] = []
        for t in path:
            p = parents[t]
            row = prompt_len - 1 if p == -1 else prompt_len + p
            if int(pred[row]) == int(draft[t]):
                acc.append(int(draft[t]))
            else:
                break
        if acc:
            brow = prompt_len + path[len(acc) - 1]
        else:
            brow = prompt_len - 1
        bonus = int(pred[brow])
        if len(acc) > len(best):
            best = acc
            best_bonus = bonus
            best_path_nodes = path[: len(acc)]
    if not best:
        best_bonus = int(pred[prompt_len - 1])
        hidden_row = prompt_len - 1
        best_node = -1
    else:
        best_node = best_path_nodes[-1]
        hidden_row = prompt_len + best_node
    return {
        "accepted_tokens": best,
        "accepted_len": len(best),
        "path": list(best_path_nodes),
        "bonus": best_bonus,
        "best_node": best_node,
        "hidden_row": hidden_row,
        "pred": pred.astype(np.int64),
    }


# --------------------------------------------------------------------------
# K1: KV-cache trim
# --------------------------------------------------------------------------
def apply_cache_slice(keys: np.ndarray, values: np.ndarray,
                      accepted_indices: Sequence[int]) -> Tuple[np.ndarray, np.ndarray, int]:
    """``new[:L] = old[idx]`` along dim 0 on copies; rest unchanged.
    ``src/gorgon/inference/kv_cache.py:89-108``."""
    idx = np.asarray(list(accepted_indices), dtype=np.int64)
    nk = keys.copy()
    nv = values.copy()
    L = idx.shape[0]
    if L > 0:
        nk[:L] = keys[idx]
        nv[:L] = values[idx]
    return nk, nv, L


def kv_trim(layers: List[Tuple[np.ndarray, np.ndarray]], idx: np.ndarray,
            lens: np.ndarray, dst_start: np.ndarray) -> List[Tuple[np.ndarray, np.ndarray]]:
    """All-layer trim-on-reject: for every layer, batch row b and kv head h,
    ``cache[b, h, dst_start[b] : dst_start[b] + lens[b]] = old[b, h, idx[b, :lens[b]]]``
    on ``[B, H, S, D]`` caches.  This is ``apply_cache_slice``
    (``src/gorgon/inference/kv_cache.py:89-108``) applied along the sequence
    axis of each (layer, b, h) slice, with the destination moved from row 0 to
    ``dst_start[b]`` so a kept prefix stays in place."""
    out = []
    for kc, vc in layers:
        nk = kc.copy()
        nv = vc.copy()
        for b in range(kc.shape[0]):
            L = int(lens[b])
            if L == 0:
                continue
            ii = np.asarray(idx[b, :L], dtype=np.int64)
            d0 = int(dst_start[b])
            nk[b, :, d0:d0 + L] = kc[b][:, ii]
            nv[b, :, d0:d0 + L] = vc[b][:, ii]
        out.append((nk, nv))
    return out


def head_topk(logits: np.ndarray, k: int) -> Tuple[np.ndarray, np.ndarray, np.ndarray, float]:
    """What one Medusa head contributes to a candidate tree
    (``src/gorgon/inference/tree_candidates.py:42-81``, ``_topk_per_head``):
    the ``min(k, V)`` largest logits and their ids in descending order (equal
    logits by ascending id), the softmax over those logits, and the entropy of
    the softmax over the whole vocabulary, ``-sum p log(p + 1e-10)``.  Computed
    in float64 from the given logits (the reference works in the logits'
    dtype)."""
    x = np.asarray(logits, dtype=np.float64).ravel()
    kk = min(int(k), x.size)
    order = np.lexsort((np.arange(x.size), -x))[:kk]
    scores = x[order]
    e = np.exp(scores - scores[0])
    probs = e / e.sum()
    p = np.exp(x - x.max())
    p /= p.sum()
    entropy = float(-(p * np.log(p + 1e-10)).sum())
    return order.astype(np.int64), scores, probs, entropy


def round_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bfloat16 (ties to even), returned as float32."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def head_logits(hidden: np.ndarray, lm_heads: Sequence[np.ndarray], round_to: Optional[str] = None) -> np.ndarray:
    """Logits of every Medusa head's last layer for one sequence
    (``MedusaHead.forward``, ``src/gorgon/models/medusa_heads.py:42-47``: a
    bias-free ``nn.Linear``): ``logits[l, v] = sum_i hidden[l, i] * W_l[v, i]``
    in float64, then as the Linear's output dtype: ``round_to`` "bf16", "f16"
    or None (float32).  ``hidden [L, H]`` holds head ``l``'s Linear input."""
    h = np.asarray(hidden, dtype=np.float64)
    out = np.stack([np.asarray(w, dtype=np.float64) @ h[l] for l, w in enumerate(lm_heads)]).astype(np.float32)
    if round_to == "bf16":
        return round_bf16(out)
    if round_to == "f16":
        return out.astype(np.float16).astype(np.float32)
    return out


def build_candidate_tree(levels, top_k: int, max_candidates: Optional[int] = None,
                         confidence_threshold: float = 0.0, use_path_confidence: bool = False,
                         entropy_weighted: bool = False) -> Tuple[List[int], List[int], List[float]]:
    """Tree assembly of ``build_candidate_tree``
    (``src/gorgon/inference/tree_candidates.py:92-245``) from the per-head
    statistics ``levels = [(ids, scores, probs, entropy), ...]`` of
    :func:`head_topk`, one entry per tree level.  Returns the nodes' tokens,
    parents (-1 for a root) and probabilities in node order.

    * Level 1 (``:149-172``): head 0's candidates in top-k order become roots,
      skipping those whose probability is below the level's threshold, until
      the budget ``max_candidates`` (``None`` = unlimited) is spent.
    * Later levels (``:175-226``): every node of the previous level, in order
      of its own logit (descending, stable) when a budget is set and in node
      order otherwise, gets one child per candidate of the level's head, in
      top-k order; a child is skipped when its probability is below the
      threshold or, with ``use_path_confidence``, when the product of
      probabilities along its path is; nodes are added until the budget is
      spent.
    * The threshold is ``confidence_threshold``, scaled by
      ``1 - entropy / log(top_k)`` (``1 - entropy`` for ``top_k <= 1``) per head
      when ``entropy_weighted`` (``:151-156``, ``:182-187``).
    """
    def threshold(entropy: float) -> float:
        if confidence_threshold > 0 and entropy_weighted:
            max_ent = math.log(top_k) if top_k > 1 else 1.0
            return confidence_threshold * (1.0 - (entropy / max_ent if max_ent > 0 else 0.0))
        return confidence_threshold

    tokens: List[int] = []
    parents: List[int] = []
    probs: List[float] = []
    path: List[float] = []
    budget = max_candidates
    if not levels:
        return tokens, parents, probs
    ids0, scores0, probs0, ent0 = levels[0]
    thr = threshold(ent0)
    level_nodes: List[Tuple[int, float]] = []
    for i in range(len(ids0)):
        if budget is not None and budget <= 0:
            break
        pr = float(probs0[i])
        if confidence_threshold > 0 and pr < thr:
            continue
        level_nodes.append((len(tokens), float(scores0[i])))
        tokens.append(int(ids0[i]))
        parents.append(-1)
        probs.append(pr)
        path.append(pr)
        if budget is not None:
            budget -= 1
    for lv in range(1, len(levels)):
        if budget is not None and budget <= 0:
            break
        ids_l, scores_l, probs_l, ent_l = levels[lv]
        thr = threshold(ent_l)
        order = (sorted(level_nodes, key=lambda x: x[1], reverse=True)
                 if max_candidates is not None else list(level_nodes))
        nxt: List[Tuple[int, float]] = []
        for pidx, _ in order:
            for i in range(len(ids_l)):
                if budget is not None and budget <= 0:
                    break
                pr = float(probs_l[i])
                if confidence_threshold > 0 and pr < thr:
                    continue
                cp = path[pidx] * pr
                if use_path_confidence and confidence_threshold > 0 and cp < thr:
                    continue
                nxt.append((len(tokens), float(scores_l[i])))
                tokens.append(int(ids_l[i]))
                parents.append(pidx)
                probs.append(pr)
                path.append(cp)
                if budget is not None:
                    budget -= 1
        level_nodes = nxt
    return tokens, parents, probs
