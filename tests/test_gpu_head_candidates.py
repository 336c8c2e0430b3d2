"""Fused Medusa heads (``gorgon_head_candidate_tree``): each head's last
Linear computed inside the statistics kernel, against the oracle.

Integer-valued inputs make every dot product exact in any summation order,
so those cases are bit-exact against the oracle -- ids, tie order (bf16
rounding of integers above 256 makes many equal logits), trees -- with
probabilities within 1e-6 and entropies within 1e-4.  Real-valued inputs
may round a logit one bf16 step away from the float64 oracle: there every
returned score must be its id's oracle logit within one bf16 step, the
scores the oracle's top-k values within one step, and the entropy within
1e-3."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import projectgorgon_b200 as G
from oracle import gorgon_oracle as O
from projectgorgon_b200.inference import (build_candidate_tree, build_candidate_trees, head_candidate_trees,
                                          medusa_head_inputs)

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _no_device_errors():
    G.device_error(clear=True)
    yield
    torch.cuda.synchronize()
    assert G.device_error(clear=True) == 0


def _int_case(B, L, H, V, seed, dtype=torch.bfloat16):
    rng = np.random.default_rng(seed)
    x = rng.integers(-3, 4, size=(B, L, H)).astype(np.float32)
    ws = [rng.integers(-2, 3, size=(V, H)).astype(np.float32) for _ in range(L)]
    xt = torch.from_numpy(x).to("cuda", dtype)
    wt = [torch.from_numpy(w).to("cuda", dtype) for w in ws]
    return x, ws, xt, wt


def _oracle_trees(x, ws, top_k, rnd, **rules):
    out = []
    for b in range(x.shape[0]):
        lg = O.head_logits(x[b], ws, rnd)
        levels = [O.head_topk(lg[l], top_k) for l in range(lg.shape[0])]
        out.append((levels, O.build_candidate_tree(levels, top_k, **rules)))
    return out


@pytest.mark.parametrize("B,L,H,V,top_k", [(1, 3, 256, 5000, 4), (2, 3, 512, 4096, 8), (3, 2, 264, 777, 32),
                                           (4, 3, 1024, 2049, 10), (1, 5, 64, 130000, 2)])
def test_fused_heads_exact_on_integer_inputs(B, L, H, V, top_k):
    x, ws, xt, wt = _int_case(B, L, H, V, seed=B * 100 + top_k)
    trees, st = head_candidate_trees(xt, wt, top_k=top_k, return_statistics=True)
    kk = min(top_k, V)
    for b, (levels, (tok, par, pr)) in enumerate(_oracle_trees(x, ws, top_k, "bf16")):
        for l, (ids, scores, probs, ent) in enumerate(levels):
            assert st.ids[b, l, :kk].tolist() == ids.tolist()
            np.testing.assert_array_equal(st.scores[b, l, :kk].cpu().numpy(), scores.astype(np.float32))
            np.testing.assert_allclose(st.probs[b, l, :kk].cpu().numpy(), probs, atol=1e-6)
            assert abs(float(st.entropy[b, l]) - ent) < 1e-4
        n = int(trees.n_nodes[b])
        assert trees.tokens[b, :n].tolist() == tok
        assert trees.parents[b, :n].tolist() == par
        np.testing.assert_allclose(trees.scores[b, :n].cpu().numpy(), pr, atol=1e-6)


@pytest.mark.parametrize("rules", [dict(max_candidates=20), dict(confidence_threshold=0.2),
                                   dict(confidence_threshold=0.05, use_path_confidence=True, entropy_weighted=True,
                                        max_candidates=30)])
def test_fused_heads_tree_rules(rules):
    x, ws, xt, wt = _int_case(2, 4, 128, 3000, seed=7)
    trees = head_candidate_trees(xt, wt, top_k=4, **rules)
    for b, (_, (tok, par, pr)) in enumerate(_oracle_trees(x, ws, 4, "bf16", **rules)):
        n = int(trees.n_nodes[b])
        assert trees.tokens[b, :n].tolist() == tok
        assert trees.parents[b, :n].tolist() == par
        np.testing.assert_allclose(trees.scores[b, :n].cpu().numpy(), pr, atol=1e-6)


def test_fused_heads_f16_and_f32_logits():
    x, ws, xt, wt = _int_case(1, 2, 64, 1000, seed=3, dtype=torch.float16)
    for logits_dtype, rnd in ((None, "f16"), (torch.float32, None)):
        _, st = head_candidate_trees(xt, wt, top_k=8, logits_dtype=logits_dtype, return_statistics=True)
        for l, (ids, scores, _, ent) in enumerate(_oracle_trees(x, ws, 8, rnd)[0][0]):
            assert st.ids[0, l].tolist() == ids.tolist()
            np.testing.assert_array_equal(st.scores[0, l].cpu().numpy(), scores.astype(np.float32))
            assert abs(float(st.entropy[0, l]) - ent) < 1e-4


def test_fused_heads_real_valued_llama_width():
    """A 4096-wide head over a 16k vocabulary, real-valued bf16."""
    B, L, H, V, k = 2, 3, 4096, 16000, 8
    g = torch.Generator(device="cuda").manual_seed(11)
    xt = torch.randn(B, L, H, device="cuda", generator=g).bfloat16()
    wt = [(torch.randn(V, H, device="cuda", generator=g) * 0.02).bfloat16() for _ in range(L)]
    _, st = head_candidate_trees(xt, wt, top_k=k, return_statistics=True)
    x = xt.double().cpu().numpy()
    ws = [w.double().cpu().numpy() for w in wt]
    for b in range(B):
        exact = O.head_logits(x[b], ws)          # float32 of the float64 sums
        for l in range(L):
            step = np.abs(exact[l]).max() * 2.0 ** -7   # one bf16 step at the top of the row
            ids = st.ids[b, l].cpu().numpy()
            sc = st.scores[b, l].cpu().numpy()
            assert np.all(np.abs(exact[l][ids] - sc) <= step)
            top = np.sort(exact[l])[::-1][:k]
            assert np.all(np.abs(np.sort(sc)[::-1] - top) <= step)
            _, _, _, ent = O.head_topk(O.round_bf16(exact[l]), k)
            assert abs(float(st.entropy[b, l]) - ent) < 1e-3


class _Block(torch.nn.Module):
    """The reference's ResidualBlock: x + SiLU(Linear(x)), zero-initialised."""

    def __init__(self, H):
        super().__init__()
        self.linear = torch.nn.Linear(H, H, bias=False)
        torch.nn.init.zeros_(self.linear.weight)

    def forward(self, x):
        return x + torch.nn.functional.silu(self.linear(x))


class _Head(torch.nn.Module):
    def __init__(self, H, V, w):
        super().__init__()
        self.norm = None
        self.blocks = torch.nn.ModuleList([_Block(H)])
        self.lm_head = torch.nn.Linear(H, V, bias=False)
        with torch.no_grad():
            self.lm_head.weight.copy_(w)

    def forward(self, x):
        for blk in self.blocks:
            x = blk(x)
        return self.lm_head(x)


def test_build_candidate_tree_fused_matches_unfused():
    H, V, L = 256, 4000, 4
    rng = np.random.default_rng(5)
    heads = torch.nn.ModuleList([_Head(H, V, torch.from_numpy(rng.integers(-2, 3, size=(V, H)).astype(np.float32)))
                                 for _ in range(L)]).to("cuda", torch.bfloat16)
    hidden = torch.from_numpy(rng.integers(-3, 4, size=(1, 1, H)).astype(np.float32)).to("cuda", torch.bfloat16)
    a = build_candidate_tree(heads, hidden, top_k=4, max_candidates=40)
    b = build_candidate_tree(heads, hidden, top_k=4, max_candidates=40, fused=True)
    assert a.parents == b.parents and a.depth == b.depth
    assert torch.equal(a.tokens, b.tokens)
    torch.testing.assert_close(a.scores, b.scores, atol=1e-6, rtol=0)
    x = medusa_head_inputs(heads, hidden)
    assert x.shape == (1, L, H) and torch.equal(x[0, 0], hidden[0, 0])
    logits = torch.stack([h(hidden)[0, 0] for h in heads])[None]
    t1 = build_candidate_trees(logits, top_k=4, max_candidates=40)
    t2 = head_candidate_trees(x, [h.lm_head.weight for h in heads], top_k=4, max_candidates=40)
    assert torch.equal(t1.tokens, t2.tokens) and torch.equal(t1.parents, t2.parents)


def test_fused_heads_rejects_what_it_cannot_run():
    x = torch.zeros(5, 2, 64, device="cuda", dtype=torch.bfloat16)
    w = [torch.zeros(100, 64, device="cuda", dtype=torch.bfloat16)] * 2
    with pytest.raises(RuntimeError, match="at most 4"):
        head_candidate_trees(x, w)
    with pytest.raises(RuntimeError, match="multiple of 8"):
        head_candidate_trees(torch.zeros(1, 2, 60, device="cuda", dtype=torch.bfloat16),
                             [torch.zeros(100, 60, device="cuda", dtype=torch.bfloat16)] * 2)
    with pytest.raises(RuntimeError, match="bf16 or f16"):
        head_candidate_trees(torch.zeros(1, 2, 64, device="cuda"), [torch.zeros(100, 64, device="cuda")] * 2)
    with pytest.raises(RuntimeError, match="levels"):
        head_candidate_trees(x[:1], w[:1])
