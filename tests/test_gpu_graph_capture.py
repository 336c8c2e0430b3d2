"""Every operator launches only on torch's current stream and takes its
workspace from torch's caching allocator, so a decode step that calls them
can be captured in a CUDA graph.  Replaying a captured call must give the
same bits as the eager call: the tensor-core attention with whole units and
with units split across CTAs (two kernels), the CUDA-core attention with its
merge kernel, and the fused verifier."""
from __future__ import annotations

import math
import random

import pytest
import torch

import projectgorgon_b200 as G
from projectgorgon_b200.trees import random_tree

pytestmark = pytest.mark.gpu


def _capture(fn):
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = fn()
    return g, out


@pytest.mark.parametrize("B,P,backend,dtype", [
    (16, 1000, "tcgen05", torch.bfloat16),   # whole units, one launch
    (1, 2048, "tcgen05", torch.bfloat16),    # units split across CTAs + merge kernel
    (2, 700, "simt", torch.float32),         # CUDA-core split-K + merge kernel
])
def test_attention_replay_is_bit_identical(B, P, backend, dtype):
    N, Hq, Hkv, D = 64, 32, 8, 128
    rng = random.Random(B + P)
    par = torch.tensor([random_tree(N, rng, 5) for _ in range(B)], device="cuda", dtype=torch.int32)
    gen = torch.Generator(device="cuda").manual_seed(P)
    s = 1.0 / math.sqrt(D)
    q = (torch.randn(B, Hq, N, D, device="cuda", generator=gen) * s).to(dtype)
    k = (torch.randn(B, Hkv, P + N, D, device="cuda", generator=gen) * s).to(dtype)
    v = (torch.randn(B, Hkv, P + N, D, device="cuda", generator=gen) * s).to(dtype)
    eager = G.fused_tree_verify(q, k, v, par, max_depth=5, backend=backend)
    g, out = _capture(lambda: G.fused_tree_verify(q, k, v, par, max_depth=5, backend=backend))
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    # new inputs in the same buffers flow through the replay
    q.mul_(2.0)
    eager2 = G.fused_tree_verify(q, k, v, par, max_depth=5, backend=backend)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager2)
    del g


def test_verifier_replay_is_bit_identical():
    B, N, V = 4, 64, 32000
    rng = random.Random(3)
    par = torch.tensor([random_tree(N, rng, 5) for _ in range(B)], device="cuda", dtype=torch.int32)
    gen = torch.Generator(device="cuda").manual_seed(3)
    logits = torch.randn(B, N + 1, V, device="cuda", generator=gen).bfloat16()
    draft = torch.randint(0, V, (B, N), device="cuda", generator=gen, dtype=torch.int32)
    eager = G.verify_tree(logits, draft, par)
    g, res = _capture(lambda: G.verify_tree(logits, draft, par))
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(res.accepted_len, eager.accepted_len)
    assert torch.equal(res.path, eager.path)
    assert torch.equal(res.bonus, eager.bonus)
    del g


def test_kv_trim_replay_moves_the_same_rows():
    """The all-layer trim, captured once and replayed on a fresh copy of the
    caches, leaves the same bits as the eager call."""
    from projectgorgon_b200.inference.kv_cache import GorgonKVCache
    B, H, S, D, Ly = 3, 4, 300, 128, 3
    gen = torch.Generator(device="cuda").manual_seed(5)
    layers = [(torch.randn(B, H, S, D, device="cuda", generator=gen).bfloat16(),
               torch.randn(B, H, S, D, device="cuda", generator=gen).bfloat16()) for _ in range(Ly)]
    orig = [(k.clone(), v.clone()) for k, v in layers]
    idx = torch.tensor([[250, 260, 270, 0], [251, 0, 0, 0], [252, 290, 0, 0]], device="cuda", dtype=torch.int32)
    lens = torch.tensor([3, 1, 2], device="cuda", dtype=torch.int32)
    cache = GorgonKVCache()
    cache.update(layers)
    cache.trim(idx, lens, dst_start=200)
    torch.cuda.synchronize()
    eager = [(k.clone(), v.clone()) for k, v in layers]
    for (k, v), (k0, v0) in zip(layers, orig):
        k.copy_(k0)
        v.copy_(v0)
    g, _ = _capture(lambda: cache.trim(idx, lens, dst_start=200))
    for (k, v), (k0, v0) in zip(layers, orig):
        k.copy_(k0)
        v.copy_(v0)
    g.replay()
    torch.cuda.synchronize()
    for (k, v), (ke, ve) in zip(layers, eager):
        assert torch.equal(k, ke) and torch.equal(v, ve)
    del g


def test_candidate_trees_replay_is_bit_identical():
    B, L, V = 4, 4, 32000
    gen = torch.Generator(device="cuda").manual_seed(6)
    logits = (torch.randn(B, L, V, device="cuda", generator=gen) * 2).bfloat16()
    eager = G.build_candidate_trees(logits, top_k=4, max_candidates=64)
    g, res = _capture(lambda: G.build_candidate_trees(logits, top_k=4, max_candidates=64))
    g.replay()
    torch.cuda.synchronize()
    assert type(res) is type(eager)
    ea = eager if isinstance(eager, (tuple, list)) else [eager]
    ra = res if isinstance(res, (tuple, list)) else [res]
    for a, b in zip(ea, ra):
        if isinstance(a, torch.Tensor):
            assert torch.equal(a, b)
    del g
