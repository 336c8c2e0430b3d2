"""The CTA-pair tcgen05 tree-attention kernel (backend "tcgen05-pair")
against the oracle: partly filled units and tiles, no prefix, a single
node, 256-node trees, f16 with a dense tree mask, log-sum-exp, batches with
several units per CTA pair, and the planner's choice on the Llama-3-8B layer.

Tolerance: bf16/f16 outputs within 2e-3 abs / 1e-2 rel of an fp32 oracle on
the same rounded inputs; log-sum-exp within 2e-3 abs of the CUDA-core
kernel's."""
from __future__ import annotations

import math
import random

import numpy as np
import pytest
import torch

import projectgorgon_b200 as G
from oracle import gorgon_oracle as O
from projectgorgon_b200.trees import best_first_tree, random_tree

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-3, 1e-2


def _np(t):
    return t.detach().float().cpu().numpy()


def _inputs(B, Hq, Hkv, N, L, D=128, dtype=torch.bfloat16, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    s = 1.0 / math.sqrt(D)
    q = (torch.randn(B, Hq, N, D, device="cuda", generator=g) * s).to(dtype)
    k = (torch.randn(B, Hkv, L, D, device="cuda", generator=g) * s).to(dtype)
    v = (torch.randn(B, Hkv, L, D, device="cuda", generator=g) * s).to(dtype)
    return q, k, v


def _trees(B, N, seed, depth=5):
    rng = random.Random(seed)
    return [random_tree(N, rng, depth) for _ in range(B)]


@pytest.fixture(autouse=True)
def _no_device_errors():
    G.device_error(clear=True)
    yield
    torch.cuda.synchronize()
    assert G.device_error(clear=True) == 0


@pytest.mark.parametrize("B,Hq,Hkv,N,P", [
    (1, 32, 8, 64, 2048),    # 8 units, prefix a multiple of the 128-key tile
    (2, 32, 8, 64, 1000),    # last tile partly past the sequence
    (1, 8, 2, 100, 300),     # 400 packed rows: a full and a partly filled unit per kv head
    (1, 2, 2, 256, 500),     # 256-node tree (8 ancestor words)
    (2, 4, 4, 64, 0),        # no prefix: one partly filled tile, one parity only
    (1, 32, 8, 1, 70),       # single node: 4 rows of a unit
    (1, 32, 8, 64, 64),      # prefix of one half tile: the tree straddles two halves
    (3, 32, 8, 64, 131),     # odd tile count per unit
])
def test_pair_matches_oracle(B, Hq, Hkv, N, P):
    pars = _trees(B, N, seed=N + P)
    q, k, v = _inputs(B, Hq, Hkv, N, P + N, seed=P)
    par_t = torch.tensor(pars, device="cuda")
    plan = G.tree_attention_plan(q, k, v, parents=par_t, max_depth=5, backend="tcgen05-pair")
    assert plan["backend"] == "tcgen05-pair" and plan["launches"] == 1 and plan["workspace_bytes"] == 0
    out = G.tree_attention(q, k, v, parents=par_t, max_depth=5, backend="tcgen05-pair")
    ref = O.tree_attention_batched(_np(q), _np(k), _np(v), parents=np.array(pars), max_depth=5)
    np.testing.assert_allclose(_np(out), ref, atol=ATOL, rtol=RTOL)


def test_pair_lse_f16_and_dense_tree_mask():
    B, Hq, Hkv, N, P = 2, 16, 4, 48, 600
    par = _trees(1, N, seed=9)[0]
    q, k, v = _inputs(B, Hq, Hkv, N, P + N, dtype=torch.float16, seed=9)
    m = G.build_tree_mask(par)
    out, lse = G.tree_attention(q, k, v, m, backend="tcgen05-pair", return_lse=True)
    _, lse_s = G.tree_attention(q, k, v, m, backend="simt", return_lse=True)
    ref = O.tree_attention_batched(_np(q), _np(k), _np(v), parents=par)
    assert out.dtype == torch.float16
    np.testing.assert_allclose(_np(out), ref, atol=ATOL, rtol=RTOL)
    np.testing.assert_allclose(_np(lse), _np(lse_s), atol=2e-3, rtol=1e-4)


def test_pair_wide_best_first_trees():
    """256-node best-first trees (top-k 4 over 4 levels), four units per
    (sequence, kv head), against the oracle."""
    B, Hq, Hkv, N, P = 2, 8, 2, 256, 700
    rng = random.Random(7)
    pars = [best_first_tree(rng, 4, 4, N)[0] for _ in range(B)]
    q, k, v = _inputs(B, Hq, Hkv, N, P + N, seed=7)
    out = G.tree_attention(q, k, v, parents=torch.tensor(pars, device="cuda"), max_depth=8,
                           backend="tcgen05-pair")
    ref = O.tree_attention_batched(_np(q), _np(k), _np(v), parents=np.array(pars), max_depth=8)
    np.testing.assert_allclose(_np(out), ref, atol=ATOL, rtol=RTOL)


def test_pair_several_units_per_pair():
    """More units than CTA pairs fit on the GPU: every pair walks several
    units, reusing its Q tile, S buffers and O accumulators; checked against
    the CUDA-core kernel over all rows and against the oracle on slices."""
    B, Hq, Hkv, N, P = 24, 32, 8, 64, 900
    pars = _trees(B, N, seed=24)
    q, k, v = _inputs(B, Hq, Hkv, N, P + N, seed=24)
    par_t = torch.tensor(pars, device="cuda")
    plan = G.tree_attention_plan(q, k, v, parents=par_t, max_depth=5, backend="tcgen05-pair")
    assert plan["splits"] < 2 * B * Hkv  # fewer pairs than units
    a = G.fused_tree_verify(q, k, v, par_t, max_depth=5, backend="tcgen05-pair")
    b = G.fused_tree_verify(q, k, v, par_t, max_depth=5, backend="simt")
    torch.testing.assert_close(a.float(), b.float(), atol=ATOL, rtol=RTOL)
    for bb, h in ((0, 0), (B - 1, Hq - 1), (11, 17)):
        ref = O.fused_tree_verify(_np(q[bb, h]), _np(k[bb, h // 4]), _np(v[bb, h // 4]), pars[bb], 5)
        np.testing.assert_allclose(_np(a[bb, h]), ref, atol=ATOL, rtol=RTOL)


def test_pair_writes_strided_output():
    """out= given as a head-major view (the layout of a head-sharded layer's
    output buffer)."""
    B, Hq, Hkv, N, P = 2, 32, 8, 64, 500
    pars = _trees(B, N, seed=3)
    q, k, v = _inputs(B, Hq, Hkv, N, P + N, seed=3)
    full = torch.empty(Hq, B, N, 128, device="cuda", dtype=torch.bfloat16)
    out = full.permute(1, 0, 2, 3)
    G.tree_attention(q, k, v, parents=torch.tensor(pars, device="cuda"), max_depth=5,
                     backend="tcgen05-pair", out=out)
    ref = O.tree_attention_batched(_np(q), _np(k), _np(v), parents=np.array(pars), max_depth=5)
    np.testing.assert_allclose(_np(out), ref, atol=ATOL, rtol=RTOL)


def test_planner_keeps_the_single_cta_kernel():
    """The pair kernel runs only when asked for (it measured slower)."""
    q, k, v = _inputs(16, 32, 8, 64, 1024)
    par = torch.tensor(_trees(16, 64, 0), device="cuda")
    assert G.tree_attention_plan(q, k, v, parents=par)["backend"] == "tcgen05"
    assert G.tree_attention_plan(q, k, v, parents=par, backend="tcgen05-pair")["backend"] == "tcgen05-pair"


def test_pair_rejects_what_it_cannot_run():
    q, k, v = _inputs(1, 32, 8, 64, 300)
    par = torch.tensor(_trees(1, 64, 0), device="cuda")
    with pytest.raises(RuntimeError):
        G.tree_attention(q, k, v, parents=par, backend="tcgen05-pair", out_dtype=torch.float32)
    with pytest.raises(RuntimeError):
        G.tree_attention(q.float(), k.float(), v.float(), parents=par, backend="tcgen05-pair")
