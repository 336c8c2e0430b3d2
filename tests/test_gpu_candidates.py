"""Device candidate-tree builder against the reference's golden trees and
the oracle.  Trees (tokens, parents) must match exactly; probabilities within
1e-6, entropies within 1e-4 (the reference's -sum p log(p + 1e-10) against the
exact entropy the kernel computes)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import projectgorgon_b200 as G
from projectgorgon_b200 import _abi
from conftest import load_golden
from oracle import gorgon_oracle as O
from projectgorgon_b200.inference import build_candidate_trees, head_statistics, max_tree_nodes

pytestmark = pytest.mark.gpu
CAND = load_golden("candidates")


@pytest.fixture(autouse=True)
def _no_device_errors():
    G.device_error(clear=True)
    yield
    torch.cuda.synchronize()
    assert G.device_error(clear=True) == 0


class _FixedHead(torch.nn.Module):
    def __init__(self, logits):
        super().__init__()
        self.register_buffer("logits", logits)

    def forward(self, hidden):
        return self.logits[None, None]


def _case(name):
    k, md, mc, pc, ew = (int(x) for x in CAND[f"{name}_params"])
    return dict(top_k=k, max_depth=None if md < 0 else md, max_candidates=None if mc < 0 else mc,
                confidence_threshold=float(CAND[f"{name}_threshold"]), use_path_confidence=bool(pc),
                entropy_weighted=bool(ew))


@pytest.mark.parametrize("name", list(CAND["names"]))
def test_candidate_tree_matches_reference_golden(name):
    c = _case(name)
    logits = torch.from_numpy(CAND[f"{name}_logits"]).cuda()
    heads = torch.nn.ModuleList([_FixedHead(logits[h]) for h in range(logits.shape[0])])
    hidden = torch.zeros(1, 1, 8, device="cuda")
    tree = G.build_candidate_tree(heads, hidden, **c)
    assert tree.depth == int(CAND[f"{name}_depth"])
    np.testing.assert_array_equal(tree.tokens.cpu().numpy(), CAND[f"{name}_tokens"])
    assert tree.parents == [int(x) for x in CAND[f"{name}_parents"]]
    np.testing.assert_allclose(tree.scores.cpu().numpy(), CAND[f"{name}_scores"], rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("name", list(CAND["names"]))
def test_head_statistics_match_reference_golden(name):
    c = _case(name)
    depth = int(CAND[f"{name}_depth"])
    logits = torch.from_numpy(CAND[f"{name}_logits"][:depth]).cuda()
    st = head_statistics(logits, c["top_k"])
    kk = CAND[f"{name}_topk_ids"].shape[1]
    np.testing.assert_array_equal(st.ids[:, :kk].cpu().numpy(), CAND[f"{name}_topk_ids"])
    np.testing.assert_array_equal(st.scores[:, :kk].cpu().numpy(), CAND[f"{name}_topk_scores"])
    np.testing.assert_allclose(st.probs[:, :kk].cpu().numpy(), CAND[f"{name}_topk_probs"], rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(st.entropy.cpu().numpy(), CAND[f"{name}_entropy"], rtol=1e-5, atol=1e-4)
    if kk < c["top_k"]:  # top_k above the vocabulary
        assert (st.ids[:, kk:] == -1).all() and (st.probs[:, kk:] == 0).all()


def _oracle_trees(logits: np.ndarray, top_k, **rules):
    out = []
    for b in range(logits.shape[0]):
        levels = [O.head_topk(logits[b, l], top_k) for l in range(logits.shape[1])]
        out.append(O.build_candidate_tree(levels, top_k, **rules))
    return out


def _check_against_oracle(lg: torch.Tensor, top_k, cap=None, **rules):
    trees = build_candidate_trees(lg, top_k=top_k, max_nodes=cap, **rules)
    ref = _oracle_trees(lg.float().cpu().numpy(), top_k, **rules)
    n = trees.n_nodes.cpu().numpy()
    toks, pars, probs = trees.tokens.cpu().numpy(), trees.parents.cpu().numpy(), trees.scores.cpu().numpy()
    for b, (rt, rp, rpr) in enumerate(ref):
        assert n[b] == len(rt), (b, n[b], len(rt))
        np.testing.assert_array_equal(toks[b, :n[b]], rt)
        np.testing.assert_array_equal(pars[b, :n[b]], rp)
        np.testing.assert_allclose(probs[b, :n[b]], rpr, rtol=1e-5, atol=1e-6)
        assert (toks[b, n[b]:] == -1).all() and (pars[b, n[b]:] == -1).all()
    return trees


RULES = [
    dict(),
    dict(max_candidates=64),
    dict(max_candidates=17),
    dict(confidence_threshold=0.17),
    dict(confidence_threshold=0.08, use_path_confidence=True),
    dict(confidence_threshold=0.3, entropy_weighted=True),
    dict(max_candidates=40, confidence_threshold=0.05, use_path_confidence=True, entropy_weighted=True),
]


@pytest.mark.parametrize("rules", RULES, ids=[str(i) for i in range(len(RULES))])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_batched_trees_match_oracle(rules, dtype):
    g = torch.Generator(device="cuda").manual_seed(len(str(rules)))
    scale = 6.0 if rules.get("entropy_weighted") else 2.5
    lg = (torch.randn(5, 4, 3001, device="cuda", generator=g) * scale).to(dtype)
    _check_against_oracle(lg, 4, **rules)


@pytest.mark.parametrize("top_k", [1, 3, 9, 17, 32])
def test_every_list_size(top_k):
    g = torch.Generator(device="cuda").manual_seed(top_k)
    lg = torch.randn(3, 2, 5000, device="cuda", generator=g) * 3
    _check_against_oracle(lg, top_k, max_candidates=300)


def test_llama3_vocabulary_bf16():
    """Four Medusa heads over a 128256-token vocabulary, 8 sequences."""
    g = torch.Generator(device="cuda").manual_seed(5)
    lg = (torch.randn(8, 4, 128256, device="cuda", generator=g) * 2).bfloat16()
    _check_against_oracle(lg, 4, max_candidates=64)
    st = head_statistics(lg, 4)
    ref = [[O.head_topk(lg[b, l].float().cpu().numpy(), 4) for l in range(4)] for b in range(8)]
    np.testing.assert_allclose(st.entropy.cpu().numpy(), [[r[3] for r in row] for row in ref], rtol=0, atol=1e-4)


def test_ties_unaligned_rows_and_masked_logits():
    """Integer logits (many ties: equal values by ascending id), an odd
    vocabulary (rows not 16-byte aligned, so the scalar path runs) and -inf
    entries."""
    g = torch.Generator(device="cuda").manual_seed(3)
    lg = torch.randint(-3, 4, (4, 3, 1001), device="cuda", generator=g).to(torch.bfloat16)
    lg[:, :, ::7] = float("-inf")
    _check_against_oracle(lg, 5, max_candidates=50)
    _check_against_oracle(lg, 5)


def test_top_k_above_vocabulary_and_tiny_rows():
    lg = torch.tensor([[[0.5, -1.0, 2.0]], [[3.0, 3.0, 1.0]]], device="cuda").repeat(1, 3, 1)
    _check_against_oracle(lg, 4)


def test_capacity_cut_sets_error_bit():
    g = torch.Generator(device="cuda").manual_seed(9)
    lg = torch.randn(2, 3, 500, device="cuda", generator=g)
    trees = build_candidate_trees(lg, top_k=4, max_nodes=30)
    torch.cuda.synchronize()
    assert G.device_error(clear=True) & _abi.ERR_CAND_CAPACITY
    full = _oracle_trees(lg.cpu().numpy(), 4)
    for b in range(2):
        assert int(trees.n_nodes[b]) == 30
        np.testing.assert_array_equal(trees.tokens[b].cpu().numpy(), full[b][0][:30])
        np.testing.assert_array_equal(trees.parents[b].cpu().numpy(), full[b][1][:30])


def test_max_tree_nodes_and_errors():
    assert max_tree_nodes(4, 4) == 340 and max_tree_nodes(4, 4, max_candidates=64) == 64
    with pytest.raises(ValueError):
        build_candidate_trees(torch.randn(2, 10), top_k=2)
    with pytest.raises(RuntimeError):
        build_candidate_trees(torch.randn(1, 2, 10, device="cuda"), top_k=33)
    with pytest.raises(RuntimeError):
        build_candidate_trees(torch.randint(0, 5, (1, 2, 10), device="cuda"), top_k=2)
