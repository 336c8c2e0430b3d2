"""Fused verifier on the GPU: bit-exact argmax, accepted length, path, bonus.

Golden cases come from the reference's own _verify_tree_candidates and
accept_draft_tokens (tests/golden/verify.npz); larger cases compare with the
oracle on the same inputs."""
from __future__ import annotations

import random

import numpy as np
import pytest
import torch

import projectgorgon_b200 as G
from conftest import load_golden
from oracle import gorgon_oracle as O
from projectgorgon_b200.trees import random_tree

pytestmark = pytest.mark.gpu
VER = load_golden("verify")


@pytest.mark.parametrize("name", list(VER["names"]))
def test_golden_tree_verification(name):
    par = [int(x) for x in VER[f"{name}_parents"]]
    logits = torch.from_numpy(VER[f"{name}_logits"]).cuda()
    draft = torch.from_numpy(VER[f"{name}_draft"]).cuda()
    pl = int(VER[f"{name}_prompt_len"])
    r = G.verify_tree(logits, draft, par, prompt_len=pl)
    acc = r.accepted_tokens(draft)[0]
    assert acc == [int(x) for x in VER[f"{name}_accepted"]]
    assert int(r.bonus) == int(VER[f"{name}_bonus"])
    assert int(r.hidden_row) == int(VER[f"{name}_hidden_row"])


@pytest.mark.parametrize("i", range(6))
def test_golden_chain_acceptance(i):
    logits = torch.from_numpy(VER[f"chain_{i}_logits"]).cuda()
    acc, rej = G.accept_draft_tokens([int(x) for x in VER[f"chain_{i}_draft"]], logits)
    assert acc == [int(x) for x in VER[f"chain_{i}_accepted"]]
    assert rej == int(VER[f"chain_{i}_rejected_at"])


def test_reference_acceptance_cases():
    draft = [1, 2, 3]
    logits = torch.tensor([[0.0, 2.0, 0.0, 0.0], [0.0, 0.0, 3.0, 0.0], [4.0, 0.0, 0.0, 0.0]],
                          device="cuda")
    assert G.accept_draft_tokens(draft, logits) == ([1, 2], 2)
    logits = torch.zeros(3, 100, device="cuda")
    logits[0, 10] = logits[1, 20] = logits[2, 30] = 10.0
    assert G.accept_draft_tokens([10, 20, 30], logits) == ([10, 20, 30], 3)
    logits = torch.zeros(3, 100, device="cuda")
    logits[0, 99] = 10.0
    assert G.accept_draft_tokens([10, 20, 30], logits) == ([], 0)


def _c5_like(B, n, V, seed, dtype=torch.bfloat16):
    """Logits N(0, 2), drafts uniform, 25% of nodes forced to match along
    random root paths; node 0 is the explicit root so drafts are nodes 1..n-1
    in the reference's prompt_len = 1 numbering."""
    rng = random.Random(seed)
    g = torch.Generator(device="cuda").manual_seed(seed)
    logits = (torch.randn(B, n, V, device="cuda", generator=g) * 2.0).to(dtype)
    pred = logits.float().argmax(-1).cpu().numpy()
    drafts, parents = [], []
    for b in range(B):
        par = random_tree(n, rng, 5)
        ref_par = [p - 1 for p in par[1:]]  # drop the explicit root
        ch = [[] for _ in range(n)]
        for i, p in enumerate(par):
            if p >= 0:
                ch[p].append(i)
        d = [rng.randrange(V) for _ in range(n - 1)]
        forced = 0
        while forced < (n - 1) // 4:
            u = 0
            while ch[u] and forced < (n - 1) // 4:
                c = rng.choice(ch[u])
                d[c - 1] = int(pred[b, u])
                forced += 1
                u = c
        drafts.append(d)
        parents.append(ref_par)
    return logits, torch.tensor(drafts, device="cuda"), torch.tensor(parents, device="cuda")


@pytest.mark.parametrize("V,dtype", [(128256, torch.bfloat16), (32000, torch.float16),
                                     (50021, torch.float32)])
def test_batched_tree_verification_bit_exact(V, dtype):
    B, n = 6, 64
    logits, draft, parents = _c5_like(B, n, V, seed=V % 97, dtype=dtype)
    r = G.verify_tree(logits, draft, parents, prompt_len=1)
    lg = logits.float().cpu().numpy()
    for b in range(B):
        ref = O.verify_tree(lg[b], draft[b].tolist(), parents[b].tolist(), 1)
        np.testing.assert_array_equal(r.pred[b].cpu().numpy(), ref["pred"][: n])
        assert int(r.accepted_len[b]) == ref["accepted_len"]
        L = ref["accepted_len"]
        assert r.path[b, :L].tolist() == ref["path"]
        assert all(x == -1 for x in r.path[b, L:].tolist())
        assert int(r.bonus[b]) == ref["bonus"]
        assert int(r.best_node[b]) == ref["best_node"]
        assert int(r.hidden_row[b]) == ref["hidden_row"]


def test_argmax_ties_and_nan_follow_torch():
    V = 4099
    logits = torch.zeros(3, V, device="cuda")
    logits[0, 17] = 5.0
    logits[0, 4000] = 5.0            # tie: first index wins
    logits[1, :] = -float("inf")     # all -inf: index 0
    logits[2, 100] = float("nan")
    logits[2, 200] = float("nan")    # NaN counts as max, first NaN wins
    r = G.verify_tree(logits, torch.tensor([17, 0], device="cuda"), [-1, 0], prompt_len=1)
    assert r.pred[:3].tolist() == torch.argmax(logits, -1).tolist() == [17, 0, 100]
    assert int(r.accepted_len) == 2


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_argmax_edge_rows_in_every_logits_type(dtype):
    """Rows that separate a chunked scan from an element-by-element one:
    ties inside one 16-byte chunk, across two chunks of the same thread
    (2048 values apart with 256 threads x 8 values) and across threads; all
    -inf; NaN anywhere beats everything and the first NaN wins; -0 equals +0;
    the maximum, or the only NaN, in the vocabulary tail (V % 8 == 3)."""
    V = 4099
    rows = torch.full((8, V), -1.0)
    rows[0, 17] = 5.0
    rows[0, 4000] = 5.0                       # tie across threads
    rows[1, :] = -float("inf")
    rows[2, 100] = float("nan")
    rows[2, 200] = float("nan")
    rows[2, 7] = 9.0
    rows[3, 2050] = -0.0
    rows[3, 9] = 0.0                          # -0 == +0: first index
    rows[4, 4098] = 7.0                       # in the tail
    rows[5, 8 * 40 + 5] = 3.0
    rows[5, 8 * 40 + 2] = 3.0                 # tie inside one chunk
    rows[6, 8 * 100 + 1] = 2.0
    rows[6, 8 * (100 + 256)] = 2.0            # tie across two chunks of one thread
    rows[7, 10] = 100.0
    rows[7, 4097] = float("nan")              # the only NaN, in the tail
    logits = rows.to(dtype).cuda()
    n = 7
    r = G.verify_tree(logits, torch.zeros(n, dtype=torch.int32, device="cuda"), [-1] + list(range(n - 1)),
                      prompt_len=1)
    want = torch.argmax(logits.float().cpu(), -1).tolist()
    assert want == [17, 0, 100, 9, 4098, 322, 801, 4097]
    assert r.pred.tolist() == want


def test_unsorted_forest_and_bad_parent():
    par = [3, -1, 1, -1, 3, 0, 0]
    V, pl = 11, 2
    g = torch.Generator().manual_seed(0)
    logits = torch.randn(pl + len(par), V, generator=g)
    pred = logits.argmax(-1)
    draft = torch.tensor([int(pred[pl + 3]), 0, int(pred[pl + 1]), int(pred[pl - 1]),
                          int(pred[pl + 3]), int(pred[pl + 0]), 5])
    r = G.verify_tree(logits.cuda(), draft.cuda(), par, prompt_len=pl)
    ref = O.verify_tree(logits.numpy(), draft.tolist(), par, pl)
    assert int(r.accepted_len) == ref["accepted_len"] and r.path[: ref["accepted_len"]].tolist() == ref["path"]
    G.device_error(clear=True)
    G.verify_tree(logits.cuda(), draft.cuda(), [3, -1, 1, -1, 3, 0, 42], prompt_len=pl)
    torch.cuda.synchronize()
    assert G.device_error(clear=True) & 4
