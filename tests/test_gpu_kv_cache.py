"""KV trim on the GPU: bit-exact against apply_cache_slice (golden) and the
all-layer oracle, including in-place gathers whose rows overlap."""
from __future__ import annotations

import random

import numpy as np
import pytest
import torch

import projectgorgon_b200 as G
from conftest import load_golden
from oracle import gorgon_oracle as O

pytestmark = pytest.mark.gpu
KV = load_golden("kv_cache")


@pytest.mark.parametrize("name", list(KV["names"]))
def test_golden_apply_cache_slice(name):
    k = torch.from_numpy(KV[f"{name}_k"]).cuda()
    v = torch.from_numpy(KV[f"{name}_v"]).cuda()
    k0, v0 = k.clone(), v.clone()
    nk, nv, L = G.apply_cache_slice(k, v, [int(x) for x in KV[f"{name}_idx"]])
    assert L == int(KV[f"{name}_len"])
    np.testing.assert_array_equal(nk.cpu().numpy(), KV[f"{name}_new_k"])
    np.testing.assert_array_equal(nv.cpu().numpy(), KV[f"{name}_new_v"])
    assert torch.equal(k, k0) and torch.equal(v, v0)


@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 128), (torch.float32, 64), (torch.float16, 5)])
def test_all_layer_in_place_trim(dtype, D):
    rng = random.Random(1)
    Lyr, B, H, P, N = 4, 5, 3, 37, 16
    S = P + N + 3
    g = torch.Generator(device="cuda").manual_seed(2)
    layers = [(torch.randn(B, H, S, D, device="cuda", generator=g).to(dtype),
               torch.randn(B, H, S, D, device="cuda", generator=g).to(dtype)) for _ in range(Lyr)]
    ref_in = [(k.float().cpu().numpy(), v.float().cpu().numpy()) for k, v in layers]
    max_len = 6
    idx = np.zeros((B, max_len), dtype=np.int32)
    lens = np.zeros(B, dtype=np.int32)
    for b in range(B):
        L = [3, 0, 6, 1, 5][b]
        path = sorted(rng.sample(range(N), L))
        if L and b == 0:
            path = [0, 2, 4]  # slot 1 <- row 2 while row 2 <- row 4
        idx[b, :L] = [P + t for t in path]
        lens[b] = L
    dst = np.full(B, P, dtype=np.int32)
    cache = G.GorgonKVCache()
    cache.update(tuple(layers))
    cache.trim(torch.from_numpy(idx).cuda(), torch.from_numpy(lens).cuda(), P)
    want = O.kv_trim(ref_in, idx, lens, dst)
    for (k, v), (wk, wv) in zip(cache.past_key_values, want):
        np.testing.assert_array_equal(k.float().cpu().numpy(), wk)
        np.testing.assert_array_equal(v.float().cpu().numpy(), wv)


@pytest.mark.parametrize("max_len", [16, 17])
def test_in_place_trim_at_the_register_path_limit(max_len):
    """16 accepted rows of 256 bytes fill the warp path's registers exactly;
    17 take the shared-memory path.  11 heads leave a partly used CTA, and
    every destination slot overlaps a later source row."""
    Lyr, B, H, D, P = 2, 3, 11, 128, 20
    S = P + 2 * max_len + 5
    g = torch.Generator(device="cuda").manual_seed(max_len)
    layers = [(torch.randn(B, H, S, D, device="cuda", generator=g).bfloat16(),
               torch.randn(B, H, S, D, device="cuda", generator=g).bfloat16()) for _ in range(Lyr)]
    ref_in = [(k.float().cpu().numpy(), v.float().cpu().numpy()) for k, v in layers]
    idx = np.zeros((B, max_len), dtype=np.int32)
    lens = np.array([max_len, max_len - 3, 1], dtype=np.int32)
    for b in range(B):
        idx[b, :lens[b]] = [P + 2 * r + 1 for r in range(lens[b])]  # row P + r <- row P + 2r + 1
    dst = np.full(B, P, dtype=np.int32)
    cache = G.GorgonKVCache()
    cache.update(tuple(layers))
    cache.trim(torch.from_numpy(idx).cuda(), torch.from_numpy(lens).cuda(), P)
    want = O.kv_trim(ref_in, idx, lens, dst)
    for (k, v), (wk, wv) in zip(cache.past_key_values, want):
        np.testing.assert_array_equal(k.float().cpu().numpy(), wk)
        np.testing.assert_array_equal(v.float().cpu().numpy(), wv)


def test_trim_from_verifier_outputs_without_host_sync():
    """verify_tree's device path feeds KVCache.trim directly (idx = P + path)."""
    B, n, V, P, H, D = 3, 8, 300, 20, 2, 16
    par = [-1, 0, 0, 1, 1, 2, 3, 6]
    logits = torch.randn(B, n + 1, V, device="cuda")
    pred = logits.argmax(-1)
    draft = torch.randint(0, V, (B, n), device="cuda")
    for b in range(B):
        for t in range(n):
            p = par[t]
            if (t + b) % 3:
                draft[b, t] = pred[b, 0 if p < 0 else p + 1]
    r = G.verify_tree(logits, draft, par, prompt_len=1)
    k = torch.randn(B, H, P + n + 1, D, device="cuda")
    v = torch.randn(B, H, P + n + 1, D, device="cuda")
    ref = [(k.cpu().numpy(), v.cpu().numpy())]
    src = torch.where(r.path >= 0, r.path + P + 1, torch.zeros_like(r.path))
    cache = G.GorgonKVCache()
    cache.update(((k, v),))
    cache.trim(src, r.accepted_len, P + 1)
    want = O.kv_trim(ref, src.cpu().numpy(), r.accepted_len.cpu().numpy(), np.full(B, P + 1))
    np.testing.assert_array_equal(cache.past_key_values[0][0].cpu().numpy(), want[0][0])


def test_out_of_range_index_is_skipped_and_flagged():
    k = torch.randn(1, 1, 8, 16, device="cuda")
    v = torch.randn(1, 1, 8, 16, device="cuda")
    k0 = k.clone()
    cache = G.GorgonKVCache()
    cache.update(((k, v),))
    G.device_error(clear=True)
    cache.trim(torch.tensor([[1, 99]], device="cuda"), torch.tensor([2], device="cuda"), 0)
    torch.cuda.synchronize()
    assert G.device_error(clear=True) & 2
    assert torch.equal(k, k0)
