"""The oracle against golden vectors produced by the reference's own code
(tests/golden/make_golden.py).  CPU only."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import load_golden, unpack_lists
from oracle import gorgon_oracle as O

MASKS = load_golden("tree_mask")
ATT = load_golden("attention")
VER = load_golden("verify")
KV = load_golden("kv_cache")


@pytest.mark.parametrize("name", list(MASKS["names"]))
@pytest.mark.parametrize("depth", [None, 1, 2, 3, 5])
def test_build_tree_mask_matches_reference(name, depth):
    par = list(MASKS[f"{name}_parents"])
    key = "none" if depth is None else str(depth)
    np.testing.assert_array_equal(O.build_tree_mask(par, depth), MASKS[f"{name}_mask_{key}"])


@pytest.mark.parametrize("name", list(MASKS["names"]))
def test_candidate_mask_and_paths_match_reference(name):
    par = list(MASKS[f"{name}_parents"])
    np.testing.assert_array_equal(O.build_tree_mask(par, 3), MASKS[f"{name}_cand_mask_d3"])
    assert O.get_tree_paths(par) == unpack_lists(MASKS, f"{name}_paths")


def test_best_first_tree_mask():
    par = list(MASKS["bestfirst256_parents"])
    assert len(par) == 256
    np.testing.assert_array_equal(O.build_tree_mask(par), MASKS["bestfirst256_mask_none"])


@pytest.mark.parametrize("name", list(ATT["names"]))
def test_tree_attention_matches_reference(name):
    q, k, v, m = (ATT[f"{name}_{x}"] for x in ("q", "k", "v", "mask"))
    got = O.tree_attention(q, k, v, m)
    np.testing.assert_allclose(got, ATT[f"{name}_out"], atol=1e-5, rtol=1e-5, equal_nan=True)


def test_masked_row_is_nan_like_torch():
    out = ATT["masked_row_nan_out"]
    assert np.isnan(out[2]).all() and not np.isnan(out[:2]).any()


@pytest.mark.parametrize("name", ["chain4_d32", "binary5_d64", "wide16_d64", "rand20_d128"])
def test_fused_walk_equals_mask_path(name):
    par = list(ATT[f"{name}_parents"])
    q, k, v, m = (ATT[f"{name}_{x}"] for x in ("q", "k", "v", "mask"))
    depth = {"chain4_d32": len(par), "binary5_d64": 3, "wide16_d64": 2, "rand20_d128": len(par)}[name]
    np.testing.assert_allclose(O.fused_tree_verify(q, k, v, par, max_depth=depth),
                               ATT[f"{name}_out"], atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("name", list(VER["names"]))
def test_verify_tree_matches_reference(name):
    par = [int(x) for x in VER[f"{name}_parents"]]
    r = O.verify_tree(VER[f"{name}_logits"], VER[f"{name}_draft"], par,
                      int(VER[f"{name}_prompt_len"]))
    assert r["accepted_tokens"] == [int(x) for x in VER[f"{name}_accepted"]]
    assert r["bonus"] == int(VER[f"{name}_bonus"])
    assert r["hidden_row"] == int(VER[f"{name}_hidden_row"])


def test_golden_verify_cases_cover_rejection_and_acceptance():
    lens = [len(VER[f"{n}_accepted"]) for n in VER["names"]]
    assert 0 in lens and max(lens) >= 3


@pytest.mark.parametrize("i", range(6))
def test_accept_draft_tokens_matches_reference(i):
    acc, rej = O.accept_draft_tokens(list(VER[f"chain_{i}_draft"]), VER[f"chain_{i}_logits"])
    assert acc == [int(x) for x in VER[f"chain_{i}_accepted"]]
    assert rej == int(VER[f"chain_{i}_rejected_at"])


@pytest.mark.parametrize("name", list(KV["names"]))
def test_apply_cache_slice_matches_reference(name):
    nk, nv, L = O.apply_cache_slice(KV[f"{name}_k"], KV[f"{name}_v"], list(KV[f"{name}_idx"]))
    assert L == int(KV[f"{name}_len"])
    np.testing.assert_array_equal(nk, KV[f"{name}_new_k"])
    np.testing.assert_array_equal(nv, KV[f"{name}_new_v"])


def test_kv_trim_equals_apply_cache_slice_per_slice():
    rng = np.random.default_rng(0)
    B, H, S, D, L = 3, 2, 10, 4, 2
    layers = [(rng.standard_normal((B, H, S, D)), rng.standard_normal((B, H, S, D))) for _ in range(L)]
    idx = np.array([[5, 7, 9], [6, 0, 0], [0, 0, 0]])
    lens = np.array([3, 1, 0])
    dst = np.array([5, 6, 2])
    out = O.kv_trim(layers, idx, lens, dst)
    for (k, v), (nk, nv) in zip(layers, out):
        for b in range(B):
            for h in range(H):
                ek, ev, _ = O.apply_cache_slice(k[b, h, dst[b]:], v[b, h, dst[b]:],
                                                [i - dst[b] for i in idx[b, :lens[b]]])
                np.testing.assert_array_equal(nk[b, h, dst[b]:], ek)
                np.testing.assert_array_equal(nv[b, h, dst[b]:], ev)
                np.testing.assert_array_equal(nk[b, h, :dst[b]], k[b, h, :dst[b]])


CAND = load_golden("candidates")


def _cand_case(name):
    k, md, mc, pc, ew = (int(x) for x in CAND[f"{name}_params"])
    return dict(top_k=k, max_depth=None if md < 0 else md, max_candidates=None if mc < 0 else mc,
                confidence_threshold=float(CAND[f"{name}_threshold"]), use_path_confidence=bool(pc),
                entropy_weighted=bool(ew))


@pytest.mark.parametrize("name", list(CAND["names"]))
def test_head_topk_matches_reference(name):
    c = _cand_case(name)
    logits = CAND[f"{name}_logits"]
    depth = int(CAND[f"{name}_depth"])
    for h in range(depth):
        ids, scores, probs, ent = O.head_topk(logits[h], c["top_k"])
        np.testing.assert_array_equal(ids, CAND[f"{name}_topk_ids"][h])
        np.testing.assert_allclose(scores, CAND[f"{name}_topk_scores"][h], rtol=0, atol=0)
        np.testing.assert_allclose(probs, CAND[f"{name}_topk_probs"][h], rtol=1e-6, atol=1e-7)
        np.testing.assert_allclose(ent, CAND[f"{name}_entropy"][h], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("name", list(CAND["names"]))
def test_candidate_tree_matches_reference(name):
    c = _cand_case(name)
    logits = CAND[f"{name}_logits"]
    depth = int(CAND[f"{name}_depth"])
    levels = [O.head_topk(logits[h], c["top_k"]) for h in range(depth)]
    toks, pars, probs = O.build_candidate_tree(
        levels, c["top_k"], max_candidates=c["max_candidates"],
        confidence_threshold=c["confidence_threshold"], use_path_confidence=c["use_path_confidence"],
        entropy_weighted=c["entropy_weighted"])
    np.testing.assert_array_equal(np.asarray(toks, dtype=np.int64), CAND[f"{name}_tokens"])
    np.testing.assert_array_equal(np.asarray(pars, dtype=np.int64), CAND[f"{name}_parents"])
    np.testing.assert_allclose(np.asarray(probs, dtype=np.float32), CAND[f"{name}_scores"], rtol=1e-6, atol=1e-7)


def test_golden_candidate_cases_cover_every_rule():
    sizes = {str(n): len(CAND[f"{n}_tokens"]) for n in CAND["names"]}
    assert sizes["all_pruned"] == 0 and sizes["budget0"] == 0
    assert sizes["k4_d4_budget20"] == 20 and sizes["k4_d4_budget64"] == 64
    assert sizes["k4_d3"] == 4 + 16 + 64
    # thresholds prune something but not everything
    for n in ("k3_threshold", "k5_threshold_entropy", "k4_threshold_path", "k4_all_rules"):
        full = sum(int(CAND[f"{n}_params"][0]) ** (l + 1) for l in range(int(CAND[f"{n}_depth"])))
        assert 0 < sizes[n] < full, n


def test_head_logits_rounding_matches_torch():
    """The oracle's bf16 / f16 rounding of a head's logits is torch's."""
    import torch
    rng = np.random.default_rng(4)
    h = rng.standard_normal((2, 64)).astype(np.float32)
    ws = [rng.standard_normal((300, 64)).astype(np.float32) for _ in range(2)]
    exact = O.head_logits(h, ws)
    ref = np.stack([w.astype(np.float64) @ h[l].astype(np.float64) for l, w in enumerate(ws)]).astype(np.float32)
    assert np.array_equal(exact, ref)
    assert np.array_equal(O.head_logits(h, ws, "bf16"), torch.from_numpy(ref).bfloat16().float().numpy())
    assert np.array_equal(O.head_logits(h, ws, "f16"), torch.from_numpy(ref).half().float().numpy())
