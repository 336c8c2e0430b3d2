"""Host logic of the Hugging Face verify-step wiring (``inference.tree_decode``)
on CPU: the step's parent array, the attention switch, and -- with the tree
attention and depth kernels replaced by the oracle's masked softmax -- that a
tree forward gives every node the logits of a plain causal forward over its
own ancestor path at positions prefix + depth.  The same checks against the
CUDA kernels are in ``test_gpu_tree_decode.py``."""
from __future__ import annotations

import random

import numpy as np
import pytest
import torch

from oracle import gorgon_oracle as O
from projectgorgon_b200.inference import tree_decode as TD
from projectgorgon_b200.trees import random_tree

transformers = pytest.importorskip("transformers")


def _oracle_attention(q, k, v, parents=None, max_depth=None, scale=None, backend="auto"):
    """[B, Hq, n, D] over k/v [B, Hkv, P + n, D]: masked softmax on
    [ones(n, P) | build_tree_mask(parents)] in fp32 (the oracle's mask)."""
    B, Hq, n, D = q.shape
    Hkv, L = k.shape[1], k.shape[2]
    P = L - n
    par = parents.reshape(-1, n) if isinstance(parents, torch.Tensor) else torch.tensor([list(parents)])
    out = torch.empty(B, Hq, n, D, dtype=q.dtype)
    for b in range(B):
        pr = par[b if par.shape[0] > 1 else 0].tolist()
        mask = np.concatenate([np.ones((n, P), bool), O.build_tree_mask(pr)], axis=1)
        m = torch.from_numpy(mask)
        kk = k[b].float().repeat_interleave(Hq // Hkv, 0)
        vv = v[b].float().repeat_interleave(Hq // Hkv, 0)
        s = (q[b].float() @ kk.transpose(1, 2)) * scale
        s = s.masked_fill(~m, float("-inf"))
        out[b] = (torch.softmax(s, -1) @ vv).to(q.dtype)
    return out


def _oracle_depths(parents):
    par = parents if parents.dim() == 2 else parents.unsqueeze(0)
    d = torch.stack([torch.from_numpy(O.build_tree_mask(p.tolist()).sum(-1) - 1) for p in par])
    return d if parents.dim() == 2 else d[0]


@pytest.fixture
def cpu_kernels(monkeypatch):
    monkeypatch.setattr(TD, "tree_attention", _oracle_attention)
    monkeypatch.setattr(TD, "tree_depths", _oracle_depths)


def _model(seed=0):
    torch.manual_seed(seed)
    cfg = transformers.LlamaConfig(vocab_size=128, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                                   num_attention_heads=4, num_key_value_heads=2, head_dim=16,
                                   max_position_embeddings=256, attn_implementation="eager")
    return transformers.LlamaForCausalLM(cfg).eval()


def _prefill(model, prompt):
    cache = transformers.DynamicCache(config=model.config)
    with torch.no_grad():
        model(input_ids=prompt, past_key_values=cache, use_cache=True)
    return cache


def test_step_parents():
    par = torch.tensor([-1, 0, 0, 1, -1], dtype=torch.int32)
    assert TD.step_parents(par).tolist() == [-1, 0, 1, 1, 2, 0]
    batched = torch.tensor([[-1, 0], [-1, -1]], dtype=torch.int32)
    assert TD.step_parents(batched).tolist() == [[-1, 0, 1], [-1, 0, 0]]


def test_attention_switch_restores_on_error():
    model = _model()
    before = model.config._attn_implementation
    with pytest.raises(ValueError):
        with TD.tree_attention_enabled(model):
            assert model.config._attn_implementation == TD.ATTN_IMPLEMENTATION
            raise ValueError("inside")
    assert model.config._attn_implementation == before


def test_tree_attention_needs_a_tree():
    q = torch.zeros(1, 4, 3, 16)
    kv = torch.zeros(1, 2, 5, 16)
    with pytest.raises(RuntimeError, match="gorgon_parents"):
        TD.gorgon_tree_attention(None, q, kv, kv, None, scaling=0.25)
    with pytest.raises(RuntimeError, match="attention mask"):
        TD.gorgon_tree_attention(None, q, kv, kv, torch.zeros(1, 1, 3, 5), scaling=0.25,
                                 gorgon_parents=torch.tensor([-1, 0, 1]))


def test_hf_cache_layers_reads_dynamic_cache():
    model = _model()
    cache = _prefill(model, torch.arange(7).unsqueeze(0))
    layers = TD.hf_cache_layers(cache)
    assert len(layers) == 2
    assert all(k.shape == (1, 2, 7, 16) and v.shape == (1, 2, 7, 16) for k, v in layers)
    assert layers[0][0] is cache.layers[0].keys


@pytest.mark.parametrize("seed", [0, 1])
def test_tree_forward_matches_ancestor_path_forwards(cpu_kernels, seed):
    """Node t's logits equal the last logits of a causal forward over the
    prefix followed by the tokens of t's root-to-t path."""
    model = _model(seed)
    rng = random.Random(seed)
    prompt = torch.tensor([[rng.randrange(128) for _ in range(11)]])
    n = 12
    parents = random_tree(n, rng, 4)
    tokens = torch.tensor([[rng.randrange(128) for _ in range(n)]])
    cache = _prefill(model, prompt)
    with torch.no_grad():
        out = TD.tree_forward(model, tokens, parents, cache)
    assert cache.get_seq_length() == 11 + n
    assert model.config._attn_implementation == "eager"
    for t in range(n):
        path = []
        x = t
        while x >= 0:
            path.append(x)
            x = parents[x]
        path.reverse()
        ref_cache = _prefill(model, prompt)
        with torch.no_grad():
            ref = model(input_ids=tokens[:, path], past_key_values=ref_cache, use_cache=True).logits[0, -1]
        torch.testing.assert_close(out.logits[0, t], ref, atol=1e-5, rtol=1e-4)


def test_chain_tree_is_a_causal_forward(cpu_kernels):
    model = _model(3)
    prompt = torch.arange(5, 14).unsqueeze(0)
    tokens = torch.tensor([[3, 1, 4, 1, 5, 9]])
    cache = _prefill(model, prompt)
    with torch.no_grad():
        out = TD.tree_forward(model, tokens, list(range(-1, 5)), cache)
        ref = model(input_ids=tokens, past_key_values=_prefill(model, prompt), use_cache=True).logits
    torch.testing.assert_close(out.logits, ref, atol=1e-5, rtol=1e-4)
