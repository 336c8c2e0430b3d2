"""Generate the golden vectors that pin the oracle to the reference.

Runs ProjectGorgon's own functions (imported unchanged from the reference's
``src/`` tree) on small seeded inputs and stores inputs and outputs as
``tests/golden/*.npz``.  It needs the reference checkout and is run by hand:

    python tests/golden/make_golden.py /path/to/ProjectGorgon

The committed ``.npz`` files are what the tests read; nothing at test time
imports the reference.

Reference functions exercised (file:line within the reference project):

* ``build_tree_mask``          src/gorgon/kernels/tree_mask.py:16-44
* ``candidate_tree_to_mask``   src/gorgon/inference/tree_candidates.py:248-279
* ``tree_attention_ref``       src/gorgon/kernels/tree_attention_ref.py:8-18
* ``accept_draft_tokens``      src/gorgon/inference/gorgon_loop.py:161-184
* ``_verify_tree_candidates``  src/gorgon/inference/gorgon_loop.py:254-392
  (driven by a fake model that returns fixed logits, the pattern of
  tests/test_benchmark_inference.py:16-72)
* ``get_tree_paths``           src/gorgon/inference/tree_candidates.py:282-311
* ``apply_cache_slice``        src/gorgon/inference/kv_cache.py:89-108
* ``build_candidate_tree``     src/gorgon/inference/tree_candidates.py:92-245
  and ``_topk_per_head`` (:42-81), driven by fake Medusa heads that return
  fixed logits
"""
from __future__ import annotations

import random
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

from projectgorgon_b200.trees import (  # noqa: E402
    best_first_tree, cartesian_tree, random_tree, reference_random_tree)


def _load_reference(root: Path):
    sys.path.insert(0, str(root / "src"))
    from gorgon.kernels.tree_mask import build_tree_mask
    from gorgon.kernels.tree_attention_ref import tree_attention_ref
    from gorgon.inference.gorgon_loop import accept_draft_tokens, _verify_tree_candidates
    from gorgon.inference.tree_candidates import (
        CandidateTree, candidate_tree_to_mask, get_tree_paths)
    from gorgon.inference.kv_cache import apply_cache_slice
    from gorgon.inference.tree_candidates import build_candidate_tree, _topk_per_head
    return dict(build_tree_mask=build_tree_mask, tree_attention_ref=tree_attention_ref,
                build_candidate_tree=build_candidate_tree, topk_per_head=_topk_per_head,
                accept_draft_tokens=accept_draft_tokens,
                verify=_verify_tree_candidates, CandidateTree=CandidateTree,
                candidate_tree_to_mask=candidate_tree_to_mask,
                get_tree_paths=get_tree_paths, apply_cache_slice=apply_cache_slice)


def _pack_lists(prefix: str, lists, store: dict) -> None:
    store[prefix + "_count"] = np.array(len(lists))
    for i, x in enumerate(lists):
        store[f"{prefix}_{i}"] = np.asarray(x, dtype=np.int64)


TREES = {
    "single": [-1],
    "chain4": [-1, 0, 1, 2],
    "binary5": [-1, 0, 0, 1, 1],
    "wide16": [-1, -1, -1, -1, 0, 0, 0, 1, 1, 1, 2, 2, 2, 3, 3, 3],
    "small3": [-1, 0, 0],
    "cartesian31": cartesian_tree(4, 2, True),
    "rand7": reference_random_tree(7, 42),
    "rand20": reference_random_tree(20, 42),
    "rand50": reference_random_tree(50, 42),
    "c2rule64": random_tree(64, random.Random(0), 5),
    "forest_unsorted": [3, -1, 1, -1, 3, 0, 0],
}


def gen_masks(ref) -> dict:
    out = {}
    names = sorted(TREES)
    out["names"] = np.array(names)
    for name in names:
        par = TREES[name]
        out[f"{name}_parents"] = np.asarray(par, dtype=np.int64)
        for depth in (None, 1, 2, 3, 5):
            key = "none" if depth is None else str(depth)
            out[f"{name}_mask_{key}"] = ref["build_tree_mask"](par, depth).numpy()
        tree = ref["CandidateTree"](tokens=torch.zeros(len(par), dtype=torch.long),
                                    parents=par, depth=3)
        out[f"{name}_cand_mask_d3"] = ref["candidate_tree_to_mask"](tree).numpy()
        _pack_lists(f"{name}_paths", ref["get_tree_paths"](tree), out)
    bf, _ = best_first_tree(random.Random(0), 4, 4, 256)
    out["bestfirst256_parents"] = np.asarray(bf, dtype=np.int64)
    out["bestfirst256_mask_none"] = ref["build_tree_mask"](bf).numpy()
    return out


def gen_attention(ref) -> dict:
    out = {}
    cases = []
    # the reference's own test (tests/test_tree_attention_ref.py:19-31)
    torch.manual_seed(0)
    q = torch.randn(3, 4); k = torch.randn(3, 4); v = torch.randn(3, 4)
    cases.append(("ref3_d4", [-1, 0, 0], q, k, v, ref["build_tree_mask"]([-1, 0, 0])))
    g = torch.Generator().manual_seed(1)
    for name, par, d, depth in (("chain4_d32", [-1, 0, 1, 2], 32, None),
                                ("binary5_d64", [-1, 0, 0, 1, 1], 64, 3),
                                ("wide16_d64", TREES["wide16"], 64, 2),
                                ("rand20_d128", TREES["rand20"], 128, None),
                                ("rand50_d64_depth3", TREES["rand50"], 64, 3)):
        n = len(par)
        q = torch.randn(n, d, generator=g); k = torch.randn(n, d, generator=g)
        v = torch.randn(n, d, generator=g)
        cases.append((name, par, q, k, v, ref["build_tree_mask"](par, depth)))
    # prefix form: [ones(n, P) | tree mask], the rectangular mask the ref accepts
    for name, par, P, d in (("prefix_c31_P40_d128", TREES["cartesian31"], 40, 128),
                            ("prefix_rand7_P9_d16", TREES["rand7"], 9, 16)):
        n = len(par)
        q = torch.randn(n, d, generator=g) / d ** 0.5
        k = torch.randn(P + n, d, generator=g) / d ** 0.5
        v = torch.randn(P + n, d, generator=g) / d ** 0.5
        m = torch.cat([torch.ones(n, P, dtype=torch.bool), ref["build_tree_mask"](par)], 1)
        cases.append((name, par, q, k, v, m))
    # a row with no visible key: torch.softmax gives NaN
    q = torch.randn(3, 8, generator=g); k = torch.randn(3, 8, generator=g)
    v = torch.randn(3, 8, generator=g)
    m = ref["build_tree_mask"]([-1, 0, 0]).clone(); m[2, :] = False
    cases.append(("masked_row_nan", [-1, 0, 0], q, k, v, m))
    out["names"] = np.array([c[0] for c in cases])
    for name, par, q, k, v, m in cases:
        out[f"{name}_parents"] = np.asarray(par, dtype=np.int64)
        out[f"{name}_q"] = q.numpy(); out[f"{name}_k"] = k.numpy(); out[f"{name}_v"] = v.numpy()
        out[f"{name}_mask"] = m.numpy()
        out[f"{name}_out"] = ref["tree_attention_ref"](q, k, v, m).numpy()
    return out


class _FakeOut:
    def __init__(self, logits, hidden):
        self.logits = logits
        self.hidden_states = (hidden,)
        self.past_key_values = None


class _FakeModel(torch.nn.Module):
    """Returns fixed logits for whatever sequence it is given; hidden state
    channel 0 holds the row index so the chosen hidden row can be read back."""

    def __init__(self, logits):
        super().__init__()
        self._logits = logits

    def forward(self, input_ids, output_hidden_states=False, use_cache=True,
                past_key_values=None):
        t = input_ids.shape[1]
        assert t == self._logits.shape[0], (t, self._logits.shape)
        hidden = torch.arange(t, dtype=torch.float32).view(1, t, 1)
        return _FakeOut(self._logits[None], hidden)


def gen_verify(ref) -> dict:
    out = {}
    rng = random.Random(7)
    g = torch.Generator().manual_seed(7)
    cases = []
    vocab = 50
    specs = [
        ("chain4_p3", TREES["chain4"], 3, 0.9),
        ("binary5_p1", TREES["binary5"], 1, 0.8),
        ("wide16_p2", TREES["wide16"], 2, 0.7),
        ("cart31_p1", cartesian_tree(4, 2, False), 1, 0.6),
        ("rand20_p4", TREES["rand20"], 4, 0.5),
        ("forest_unsorted_p2", TREES["forest_unsorted"], 2, 0.7),
        ("none_accepted_p2", TREES["binary5"], 2, 0.0),
        ("ties_p1", TREES["wide16"], 1, 0.5),
    ]
    for name, par, prompt_len, force in specs:
        n = len(par)
        rows = prompt_len + n
        logits = torch.randn(rows, vocab, generator=g)
        if name.startswith("ties"):
            logits = torch.randint(0, 3, (rows, vocab), generator=g).float()
        pred = logits.argmax(-1)
        draft = torch.randint(0, vocab, (n,), generator=g)
        for t in range(n):
            p = par[t]
            row = prompt_len - 1 if p == -1 else prompt_len + p
            if rng.random() < force:
                draft[t] = pred[row]
        cases.append((name, par, prompt_len, logits, draft))
    out["names"] = np.array([c[0] for c in cases])
    for name, par, prompt_len, logits, draft in cases:
        tree = ref["CandidateTree"](tokens=draft.clone(), parents=list(par), depth=5)
        input_ids = torch.zeros(1, prompt_len, dtype=torch.long)
        model = _FakeModel(logits)
        best, bonus, hidden, _ = ref["verify"](model, input_ids, tree, past_key_values=None)
        out[f"{name}_parents"] = np.asarray(par, dtype=np.int64)
        out[f"{name}_prompt_len"] = np.array(prompt_len)
        out[f"{name}_logits"] = logits.numpy()
        out[f"{name}_draft"] = draft.numpy().astype(np.int64)
        out[f"{name}_accepted"] = np.asarray(best, dtype=np.int64)
        out[f"{name}_bonus"] = np.array(bonus)
        out[f"{name}_hidden_row"] = np.array(int(hidden.reshape(-1)[0].item()))
    # greedy chain acceptance
    chain = []
    for i in range(6):
        L = 1 + i
        logits = torch.randn(L, 20, generator=g)
        draft = logits.argmax(-1).tolist()
        if i % 2 == 1:
            draft[i // 2] = (draft[i // 2] + 1) % 20
        acc, rej = ref["accept_draft_tokens"](draft, logits)
        chain.append((logits, draft, acc, rej))
    out["chain_count"] = np.array(len(chain))
    for i, (logits, draft, acc, rej) in enumerate(chain):
        out[f"chain_{i}_logits"] = logits.numpy()
        out[f"chain_{i}_draft"] = np.asarray(draft, dtype=np.int64)
        out[f"chain_{i}_accepted"] = np.asarray(acc, dtype=np.int64)
        out[f"chain_{i}_rejected_at"] = np.array(rej)
    return out


def gen_kv(ref) -> dict:
    out = {}
    keys = torch.tensor([10, 11, 12, 13, 14], dtype=torch.float32)
    values = torch.tensor([110, 111, 112, 113, 114], dtype=torch.float32)
    cases = [("ref_1d", keys, values, [0, 2, 4])]
    g = torch.Generator().manual_seed(3)
    k2 = torch.randn(12, 8, generator=g); v2 = torch.randn(12, 8, generator=g)
    cases.append(("rows_overlap", k2, v2, [0, 2, 4, 5, 9]))
    cases.append(("empty", k2, v2, []))
    cases.append(("reverse", k2, v2, [11, 7, 3]))
    out["names"] = np.array([c[0] for c in cases])
    for name, k, v, idx in cases:
        nk, nv, L = ref["apply_cache_slice"](k, v, idx)
        out[f"{name}_k"] = k.numpy(); out[f"{name}_v"] = v.numpy()
        out[f"{name}_idx"] = np.asarray(idx, dtype=np.int64)
        out[f"{name}_new_k"] = nk.numpy(); out[f"{name}_new_v"] = nv.numpy()
        out[f"{name}_len"] = np.array(L)
    return out


# name, heads, vocab, top_k, max_depth, max_candidates, threshold, path_conf, entropy_w, sigma
CAND_CASES = [
    ("k4_d3", 3, 64, 4, None, None, 0.0, False, False, 2.0),
    ("k4_d4_budget20", 4, 64, 4, None, 20, 0.0, False, False, 2.0),
    ("k4_d4_budget64", 4, 200, 4, None, 64, 0.0, False, False, 2.0),
    ("k3_threshold", 3, 100, 3, None, None, 0.3, False, False, 1.0),
    ("k5_threshold_entropy", 4, 100, 5, None, None, 0.4, False, True, 5.0),
    ("k4_threshold_path", 4, 100, 4, None, None, 0.05, True, False, 2.0),
    ("k4_all_rules", 4, 150, 4, None, 30, 0.1, True, True, 2.5),
    ("k1_d5", 5, 40, 1, None, None, 0.0, False, False, 1.0),
    ("k8_d2", 2, 300, 8, None, None, 0.0, False, False, 3.0),
    ("max_depth2_of4", 4, 64, 4, 2, None, 0.0, False, False, 2.0),
    ("all_pruned", 3, 64, 4, None, None, 0.99, False, False, 0.1),
    ("budget0", 3, 64, 4, None, 0, 0.0, False, False, 2.0),
    ("k_above_vocab", 2, 3, 4, None, None, 0.0, False, False, 1.0),
    ("k4_d3_budget7_threshold", 3, 80, 4, None, 7, 0.2, False, False, 1.2),
]


class _FixedHead(torch.nn.Module):
    """A Medusa head stand-in that returns fixed logits (1, 1, vocab)."""

    def __init__(self, logits):
        super().__init__()
        self.register_buffer("logits", logits)

    def forward(self, hidden):
        return self.logits[None, None]


def gen_candidates(ref) -> dict:
    out = {"names": np.array([c[0] for c in CAND_CASES])}
    g = torch.Generator().manual_seed(11)
    hidden = torch.zeros(1, 1, 8)
    for name, nh, vocab, k, md, mc, thr, pc, ew, sigma in CAND_CASES:
        logits = torch.randn(nh, vocab, generator=g) * sigma
        heads = torch.nn.ModuleList([_FixedHead(logits[h]) for h in range(nh)])
        tree = ref["build_candidate_tree"](heads, hidden, top_k=k, max_depth=md, max_candidates=mc,
                                           confidence_threshold=thr, use_path_confidence=pc,
                                           entropy_weighted=ew)
        depth = min(md or nh, nh)
        stats = ref["topk_per_head"](heads[:depth], hidden, k)
        out[f"{name}_logits"] = logits.numpy()
        out[f"{name}_params"] = np.array([k, -1 if md is None else md, -1 if mc is None else mc,
                                          int(pc), int(ew)], dtype=np.int64)
        out[f"{name}_threshold"] = np.array(thr, dtype=np.float64)
        out[f"{name}_tokens"] = tree.tokens.numpy().astype(np.int64)
        out[f"{name}_parents"] = np.asarray(tree.parents, dtype=np.int64)
        out[f"{name}_depth"] = np.array(tree.depth)
        out[f"{name}_scores"] = tree.scores.numpy().astype(np.float32)
        out[f"{name}_topk_ids"] = np.stack([s.ids.numpy() for s in stats]).astype(np.int64)
        out[f"{name}_topk_scores"] = np.stack([s.scores.numpy() for s in stats]).astype(np.float32)
        out[f"{name}_topk_probs"] = np.stack([s.probs.numpy() for s in stats]).astype(np.float32)
        out[f"{name}_entropy"] = np.array([s.entropy for s in stats], dtype=np.float64)
    return out


def main() -> None:
    root = Path(sys.argv[1]) if len(sys.argv) > 1 else None
    if root is None or not (root / "src" / "gorgon").is_dir():
        raise SystemExit("usage: make_golden.py <ProjectGorgon checkout>")
    ref = _load_reference(root)
    for name, fn in (("tree_mask", gen_masks), ("attention", gen_attention),
                     ("verify", gen_verify), ("kv_cache", gen_kv), ("candidates", gen_candidates)):
        data = fn(ref)
        np.savez_compressed(HERE / f"{name}.npz", **data)
        print(name, len(data), "arrays")


if __name__ == "__main__":
    main()
