"""Host-side logic that needs no GPU: tree generators, argument handling of
the Python operator surface, exception types."""
from __future__ import annotations

import random

import pytest
import torch

import projectgorgon_b200 as G
from projectgorgon_b200 import trees
from oracle import gorgon_oracle as O


def test_random_tree_rule():
    par = trees.random_tree(64, random.Random(0), 5)
    assert par[0] == -1 and all(0 <= p < i for i, p in enumerate(par) if i)
    assert max(trees.tree_depths(par)) <= 5


def test_cartesian_tree_has_31_nodes():
    par = trees.cartesian_tree(4, 2, True)
    assert len(par) == 31 and par[:7] == [-1, 0, 0, 1, 1, 2, 2]
    assert max(trees.tree_depths(par)) == 4


def test_best_first_tree_closed_under_ancestors():
    par, cum = trees.best_first_tree(random.Random(1), 4, 4, 256)
    assert len(par) == 256 and par[0] == -1
    assert all(p < i for i, p in enumerate(par))
    assert max(trees.tree_depths(par)) <= 4


def test_reference_random_tree_matches_benchmark_rule():
    rng = random.Random(5)
    expect = [-1] + [rng.randrange(0, i) for i in range(1, 9)]
    assert trees.reference_random_tree(9, 5) == expect


@pytest.mark.parametrize("fn", [G.tree_attention_cuda, G.tree_attention_triton])
def test_host_tensors_raise_value_error(fn):
    q = torch.randn(3, 4)
    with pytest.raises(ValueError):
        fn(q, q, q, torch.ones(3, 3, dtype=torch.bool))


def test_fused_and_verify_reject_host_tensors():
    q = torch.randn(3, 4)
    with pytest.raises(ValueError):
        G.fused_tree_verify(q, q, q, [-1, 0, 0])
    with pytest.raises(ValueError):
        G.verify_tree(torch.randn(4, 10), torch.zeros(3, dtype=torch.long), [-1, 0, 0])
    with pytest.raises(ValueError):
        G.apply_cache_slice(torch.zeros(5), torch.zeros(5), [0, 2])
    with pytest.raises(ValueError):
        G.accept_draft_tokens([1, 2], torch.randn(2, 5))


def test_candidate_builders_reject_host_tensors():
    from projectgorgon_b200.inference import build_candidate_trees, head_candidate_trees
    with pytest.raises(ValueError):
        build_candidate_trees(torch.randn(1, 2, 100))
    x = torch.zeros(1, 2, 64, dtype=torch.bfloat16)
    w = [torch.zeros(100, 64, dtype=torch.bfloat16)] * 2
    with pytest.raises(ValueError):
        head_candidate_trees(x, w)


def test_verify_oracle_preorder_rule_on_random_trees():
    """The kernel's selection rule (deepest accepted node, first in preorder)
    equals the reference's path loop, checked on the oracle."""
    rng = random.Random(3)
    import numpy as np
    for trial in range(200):
        n = rng.randint(1, 24)
        par = [-1 if i == 0 or rng.random() < 0.15 else rng.randrange(0, i) for i in range(n)]
        V = 6
        logits = np.array([[rng.random() for _ in range(V)] for _ in range(n + 2)])
        draft = [rng.randrange(V) for _ in range(n)]
        pl = 2
        ref = O.verify_tree(logits, draft, par, pl)
        pred = ref["pred"]
        acc_depth = {}
        depth = trees.tree_depths(par)
        for t in range(n):
            u, ok = t, True
            while True:
                p = par[u]
                row = pl - 1 if p < 0 else pl + p
                if pred[row] != draft[u]:
                    ok = False
                    break
                if p < 0:
                    break
                u = p
            if ok:
                acc_depth[t] = depth[t]
        if not acc_depth:
            assert ref["best_node"] == -1
            continue
        bd = max(acc_depth.values())
        cands = [t for t, d in acc_depth.items() if d == bd]
        order = [p[-1] for p in O.get_tree_paths(par)]
        # preorder position of each node
        pre = []
        def dfs(u, ch):
            pre.append(u)
            for c in ch[u]:
                dfs(c, ch)
        ch = [[] for _ in range(n)]
        for i, p in enumerate(par):
            if p >= 0:
                ch[p].append(i)
        for r in [i for i, p in enumerate(par) if p == -1]:
            dfs(r, ch)
        win = min(cands, key=pre.index)
        assert ref["best_node"] == win, (par, draft)
