"""The verify step wired into a Hugging Face decoder (``inference.tree_decode``)
on the CUDA kernels: every attention layer runs the tree attention, the
verifier picks the path and the all-layer trim edits the model's own
``DynamicCache``.

The comparison is the model itself with its stock causal attention (SDPA):
a tree node's logits are those of a causal forward over the prefix and the
node's root-to-node path, and after a step the cache holds what a causal
forward of the accepted tokens leaves.  Tolerances: fp32 (CUDA-core path)
1e-4 relative; bf16 (tcgen05 path) 2e-2 relative in the Frobenius norm."""
from __future__ import annotations

import random

import pytest
import torch

import projectgorgon_b200 as G
from projectgorgon_b200.inference import tree_decode as TD
from projectgorgon_b200.trees import random_tree

pytestmark = pytest.mark.gpu
transformers = pytest.importorskip("transformers")

VOCAB, HQ, HKV, D = 1024, 8, 2, 128
REL = {torch.float32: 1e-4, torch.bfloat16: 2e-2}


def _model(dtype, seed=0):
    torch.manual_seed(seed)
    cfg = transformers.LlamaConfig(vocab_size=VOCAB, hidden_size=HQ * D, intermediate_size=2048,
                                   num_hidden_layers=2, num_attention_heads=HQ, num_key_value_heads=HKV,
                                   head_dim=D, max_position_embeddings=4096, attn_implementation="sdpa")
    return transformers.LlamaForCausalLM(cfg).to(device="cuda", dtype=dtype).eval()


def _prefill(model, prompt):
    cache = transformers.DynamicCache(config=model.config)
    with torch.no_grad():
        model(input_ids=prompt, past_key_values=cache, use_cache=True)
    return cache


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


def _path(parents, t):
    out = []
    while t >= 0:
        out.append(t)
        t = parents[t]
    return out[::-1]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_tree_forward_matches_causal_path_forwards(dtype):
    model = _model(dtype)
    rng = random.Random(1)
    P, n = 200, 64
    prompt = torch.tensor([[rng.randrange(VOCAB) for _ in range(P)]], device="cuda")
    parents = random_tree(n, rng, 5)
    tokens = torch.tensor([[rng.randrange(VOCAB) for _ in range(n)]], device="cuda")
    if dtype == torch.bfloat16:  # this shape runs on the tensor-core kernel
        q = torch.empty(1, HQ, n, D, device="cuda", dtype=dtype)
        kv = torch.empty(1, HKV, P + n, D, device="cuda", dtype=dtype)
        assert G.tree_attention_plan(q, kv, kv, parents=parents)["backend"] == "tcgen05"
    cache = _prefill(model, prompt)
    with torch.no_grad():
        out = TD.tree_forward(model, tokens, parents, cache)
    assert cache.get_seq_length() == P + n
    assert model.config._attn_implementation == "sdpa"
    leaves = [t for t in range(n) if t not in parents]
    for t in sorted(leaves, key=lambda x: -len(_path(parents, x)))[:4] + [0]:
        path = _path(parents, t)
        with torch.no_grad():
            ref = model(input_ids=tokens[:, path], past_key_values=_prefill(model, prompt),
                        use_cache=True).logits[0]
        # every node on the path: its tree row against its causal row
        assert _rel(out.logits[0, path], ref) < REL[dtype], (t, path)


def _greedy(model, prompt, last, steps):
    cache = _prefill(model, prompt)
    toks, cur = [], last
    with torch.no_grad():
        for _ in range(steps):
            lg = model(input_ids=torch.tensor([[cur]], device="cuda"), past_key_values=cache, use_cache=True).logits
            cur = int(lg[0, -1].argmax())
            toks.append(cur)
    return toks


def test_verify_step_accepts_the_greedy_branch_and_trims_the_cache():
    """fp32: a tree whose first branch is the model's greedy continuation
    (decoys elsewhere) accepts exactly that branch; the cache afterwards is
    the causal cache of prompt + last token + accepted tokens, and decoding
    continues from it as from the causal one."""
    model = _model(torch.float32, seed=2)
    rng = random.Random(2)
    P = 150
    prompt = torch.tensor([[rng.randrange(VOCAB) for _ in range(P)]], device="cuda")
    last = rng.randrange(VOCAB)
    g = _greedy(model, prompt, last, 4)

    def decoy(avoid):
        while True:
            x = rng.randrange(VOCAB)
            if x not in avoid:
                return x
    # level 1: g0 + two decoys; under g0: g1 + decoy; under g1: g2 + decoy; under decoys: anything
    draft = [g[0], decoy(g), decoy(g), g[1], decoy(g), g[2], decoy(g), decoy(g), decoy(g)]
    parents = [-1, -1, -1, 0, 0, 3, 3, 1, 2]
    cache = _prefill(model, prompt)
    with torch.no_grad():
        res = TD.tree_verify_step(model, cache, last, torch.tensor(draft, device="cuda"), parents)
    assert res.accepted == g[:3]
    assert res.verify.path[:3].tolist() == [0, 3, 5]
    assert res.bonus == g[3]
    assert res.seq_len == P + 1 + 3 == cache.get_seq_length()
    ref = _prefill(model, torch.cat([prompt, torch.tensor([[last] + g[:3]], device="cuda")], dim=1))
    for (k, v), (rk, rv) in zip(TD.hf_cache_layers(cache), TD.hf_cache_layers(ref)):
        assert _rel(k, rk) < 1e-4 and _rel(v, rv) < 1e-4
    with torch.no_grad():
        nxt = model(input_ids=torch.tensor([[res.bonus]], device="cuda"), past_key_values=cache, use_cache=True)
        nref = model(input_ids=torch.tensor([[res.bonus]], device="cuda"), past_key_values=ref, use_cache=True)
    assert _rel(nxt.logits, nref.logits) < 1e-4


@pytest.mark.parametrize("seed", [0, 5])
def test_verify_step_bf16_is_consistent(seed, monkeypatch):
    """bf16 on the tensor-core path: the accepted path follows the step's own
    argmaxes, the bonus is the argmax after it, and the cache rows after the
    last token are the accepted nodes' K/V rows of the verify forward, moved
    bit for bit (the cache is copied just before the trim)."""
    model = _model(torch.bfloat16, seed=seed)
    rng = random.Random(seed)
    P, n = 300, 47
    prompt = torch.tensor([[rng.randrange(VOCAB) for _ in range(P)]], device="cuda")
    last = rng.randrange(VOCAB)
    g = _greedy(model, prompt, last, 3)
    parents = random_tree(n, rng, 4)
    draft = [rng.randrange(VOCAB) for _ in range(n)]
    # put the greedy chain on the first root-to-leaf path
    chain = [t for t in range(n) if parents[t] == -1][:1]
    while len(chain) < 3:
        kids = [t for t in range(n) if parents[t] == chain[-1]]
        if not kids:
            break
        chain.append(kids[0])
    for i, t in enumerate(chain):
        draft[t] = g[i]
    before = {}
    trim = TD.trim_hf_cache

    def spy(cache, src, lens, dst):
        before["kv"] = [(k.clone(), v.clone()) for k, v in TD.hf_cache_layers(cache)]
        return trim(cache, src, lens, dst)

    monkeypatch.setattr(TD, "trim_hf_cache", spy)
    cache = _prefill(model, prompt)
    with torch.no_grad():
        res = TD.tree_verify_step(model, cache, last, torch.tensor(draft, device="cuda"), parents,
                                  backend="tcgen05")
    pred = res.logits[0].float().argmax(-1).tolist()
    a = len(res.accepted)
    path = res.verify.path[:a].tolist()
    prev = -1
    for t in path:
        assert parents[t] == prev
        assert draft[t] == pred[0 if prev < 0 else 1 + prev]
        prev = t
    assert res.bonus == pred[0 if prev < 0 else 1 + prev]
    assert res.seq_len == P + 1 + a == cache.get_seq_length()
    rows = [P] + [P + 1 + t for t in path]
    for (k, v), (bk, bv) in zip(TD.hf_cache_layers(cache), before["kv"]):
        assert bk.shape[2] == P + 1 + n
        torch.testing.assert_close(k[:, :, :P], bk[:, :, :P], atol=0, rtol=0)
        torch.testing.assert_close(k[:, :, P:], bk[:, :, rows], atol=0, rtol=0)
        torch.testing.assert_close(v[:, :, P:], bv[:, :, rows], atol=0, rtol=0)
