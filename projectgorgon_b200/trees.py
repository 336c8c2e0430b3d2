"""Candidate-tree shapes used by the verify path's workloads and tests.

A tree is a ``parents`` list in the reference's flat form
(``src/gorgon/inference/tree_candidates.py:17-30``): node ``i``'s parent is
``parents[i]`` and ``-1`` marks a root.  All generators here emit parents before
children (level order), as ``build_candidate_tree`` does
(``tree_candidates.py:158-227``).
"""
from __future__ import annotations

import heapq
import random
from typing import List, Tuple

__all__ = ["random_tree", "cartesian_tree", "best_first_tree", "tree_depths",
           "reference_random_tree"]


def reference_random_tree(n: int, seed: int) -> List[int]:
    """``parents[i] = randrange(0, i)`` from ``random.Random(seed)``: the tree of
    ``scripts/benchmark_speed.py:31-36``."""
    rng = random.Random(seed)
    parents = [-1]
    for i in range(1, n):
        parents.append(rng.randrange(0, i))
    return parents[:n]


def random_tree(n: int, rng: random.Random, max_depth: int = 5) -> List[int]:
    """Node 0 is the root; node ``i >= 1`` picks its parent uniformly among the
    earlier nodes whose depth is below ``max_depth`` (root depth 0), so no node
    is more than ``max_depth`` hops from the root."""
    parents = [-1]
    depth = [0]
    eligible = [0]
    for i in range(1, n):
        p = eligible[rng.randrange(len(eligible))]
        parents.append(p)
        depth.append(depth[p] + 1)
        if depth[-1] < max_depth:
            eligible.append(i)
    return parents


def cartesian_tree(num_heads: int = 4, top_k: int = 2, with_root: bool = True) -> List[int]:
    """Full Cartesian product of ``num_heads`` levels of ``top_k`` candidates
    in level order, children of a parent contiguous.  With ``with_root`` a
    single root node 0 sits above the first level (4 heads x top_k 2 gives
    1 + 2 + 4 + 8 + 16 = 31 nodes)."""
    parents: List[int] = []
    if with_root:
        parents.append(-1)
        frontier = [0]
    else:
        frontier = [-1]
    for _ in range(num_heads):
        nxt = []
        for p in frontier:
            for _ in range(top_k):
                parents.append(p)
                nxt.append(len(parents) - 1)
        frontier = nxt
    return parents


def best_first_tree(rng: random.Random, num_heads: int = 4, top_k: int = 4,
                    max_candidates: int = 256) -> Tuple[List[int], List[float]]:
    """Root plus a ``top_k``-ary tree over ``num_heads`` levels, pruned to
    ``max_candidates`` nodes (root included) by best-first expansion on the
    cumulative log-probability, each node's own log-prob drawn N(0, 1).  The
    kept set is closed under ancestors; it is returned in level order with the
    cumulative log-probs."""
    # full tree: node -> (parent, level, logp)
    full_par = [-1]
    full_lvl = [0]
    full_cum = [0.0]
    frontier = [0]
    for lvl in range(1, num_heads + 1):
        nxt = []
        for p in frontier:
            for _ in range(top_k):
                full_par.append(p)
                full_lvl.append(lvl)
                full_cum.append(full_cum[p] + rng.gauss(0.0, 1.0))
                nxt.append(len(full_par) - 1)
        frontier = nxt
    children = [[] for _ in full_par]
    for i, p in enumerate(full_par):
        if p >= 0:
            children[p].append(i)
    kept = [0]
    heap = [(-full_cum[c], c) for c in children[0]]
    heapq.heapify(heap)
    while heap and len(kept) < max_candidates:
        _, u = heapq.heappop(heap)
        kept.append(u)
        for c in children[u]:
            heapq.heappush(heap, (-full_cum[c], c))
    kept.sort(key=lambda u: (full_lvl[u], u))
    new_id = {u: i for i, u in enumerate(kept)}
    parents = [-1 if full_par[u] < 0 else new_id[full_par[u]] for u in kept]
    cum = [full_cum[u] for u in kept]
    return parents, cum


def tree_depths(parents: List[int]) -> List[int]:
    """Hop depth of every node (roots are 0); parents must precede children."""
    d = []
    for i, p in enumerate(parents):
        d.append(0 if p < 0 else d[p] + 1)
    return d
