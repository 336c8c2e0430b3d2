"""The tcgen05 tree-attention kernel against the oracle (small shapes) and
against the CUDA-core kernel (large shapes), forcing backend="tcgen05".

Tolerance: bf16/f16 outputs within 2e-3 abs / 1e-2 rel of an fp32 oracle on
the same rounded inputs."""
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
    (1, 32, 8, 64, 2048),    # 2 M-tiles, pairs split across many CTAs
    (2, 32, 8, 64, 1000),    # prefix not a multiple of the 64-row tile
    (1, 4, 1, 7, 130),       # one partly filled M-tile
    (1, 8, 2, 100, 300),     # 400 packed rows: two query groups
    (1, 2, 2, 256, 500),     # 256-node tree (8 ancestor words)
    (2, 4, 4, 64, 0),        # no prefix
    (1, 32, 8, 1, 70),       # single node
])
def test_tc_matches_oracle(B, Hq, Hkv, N, P):
    pars = _trees(B, N, seed=N + P)
    q, k, v = _inputs(B, Hq, Hkv, N, P + N, seed=P)
    par_t = torch.tensor(pars, device="cuda")
    plan = G.tree_attention_plan(q, k, v, parents=par_t, max_depth=5, backend="tcgen05")
    assert plan["backend"] == "tcgen05"
    out = G.tree_attention(q, k, v, parents=par_t, max_depth=5, backend="tcgen05")
    ref = O.tree_attention_batched(_np(q), _np(k), _np(v), parents=np.array(pars), max_depth=5)
    np.testing.assert_allclose(_np(out), ref, atol=ATOL, rtol=RTOL)


def test_tc_lse_and_fp32_output():
    B, Hq, Hkv, N, P = 2, 8, 2, 40, 777
    pars = _trees(B, N, seed=5)
    q, k, v = _inputs(B, Hq, Hkv, N, P + N, seed=5)
    out, lse = G.tree_attention(q, k, v, parents=torch.tensor(pars, device="cuda"), max_depth=5,
                                backend="tcgen05", out_dtype=torch.float32, return_lse=True)
    _, lse_s = G.tree_attention(q, k, v, parents=torch.tensor(pars, device="cuda"), max_depth=5,
                                backend="simt", return_lse=True)
    ref = O.tree_attention_batched(_np(q), _np(k), _np(v), parents=np.array(pars), max_depth=5)
    assert out.dtype == torch.float32
    np.testing.assert_allclose(_np(out), ref, atol=ATOL, rtol=RTOL)
    np.testing.assert_allclose(_np(lse), _np(lse_s), atol=2e-3, rtol=1e-4)


def test_tc_float16_and_dense_tree_mask():
    B, Hq, Hkv, N, P = 1, 16, 4, 48, 600
    par = _trees(1, N, seed=9)[0]
    q, k, v = _inputs(B, Hq, Hkv, N, P + N, dtype=torch.float16, seed=9)
    m = G.build_tree_mask(par)
    out = G.tree_attention(q, k, v, m, backend="tcgen05")
    ref = O.tree_attention_batched(_np(q), _np(k), _np(v), parents=par)
    np.testing.assert_allclose(_np(out), ref, atol=ATOL, rtol=RTOL)


def test_tc_ragged_cu_seqlens():
    rng = random.Random(11)
    B, Hq, Hkv, N, D = 5, 32, 8, 64, 128
    Ls = [rng.randint(64, 3000) + N for _ in range(B)]
    cu = np.concatenate([[0], np.cumsum(Ls)]).astype(np.int32)
    pars = _trees(B, N, seed=11)
    g = torch.Generator(device="cuda").manual_seed(11)
    s = 1 / math.sqrt(D)
    q = (torch.randn(B, Hq, N, D, device="cuda", generator=g) * s).bfloat16()
    kp = (torch.randn(int(cu[-1]), Hkv, D, device="cuda", generator=g) * s).bfloat16()
    vp = (torch.randn(int(cu[-1]), Hkv, D, device="cuda", generator=g) * s).bfloat16()
    kw = dict(parents=torch.tensor(pars, device="cuda"), max_depth=5,
              cu_seqlens=torch.from_numpy(cu).cuda(), max_seqlen=max(Ls))
    assert G.tree_attention_plan(q, kp, vp, **kw, backend="tcgen05")["backend"] == "tcgen05"
    out = G.tree_attention(q, kp, vp, **kw, backend="tcgen05")
    for b in range(B):
        kb = _np(kp[cu[b]:cu[b + 1]]).transpose(1, 0, 2)[None]
        vb = _np(vp[cu[b]:cu[b + 1]]).transpose(1, 0, 2)[None]
        ref = O.tree_attention_batched(_np(q[b:b + 1]), kb, vb, parents=pars[b], max_depth=5)
        np.testing.assert_allclose(_np(out[b:b + 1]), ref, atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("B,P", [(16, 8192), (3, 5000)])
def test_tc_matches_simt_at_scale(B, P):
    """Llama-3-8B shape (32 q / 8 kv heads, d 128, 64-node trees): the
    tensor-core kernel against the CUDA-core kernel on the same inputs."""
    N = 64
    pars = torch.tensor(_trees(B, N, seed=B), device="cuda")
    q, k, v = _inputs(B, 32, 8, N, P + N, seed=B)
    a = G.fused_tree_verify(q, k, v, pars, max_depth=5, backend="tcgen05")
    b = G.fused_tree_verify(q, k, v, pars, max_depth=5, backend="simt")
    torch.testing.assert_close(a.float(), b.float(), atol=ATOL, rtol=RTOL)


def test_tc_wide_best_first_tree():
    """256-node best-first tree (top-k 4 over 4 levels), one kv head."""
    par, _ = best_first_tree(random.Random(0), 4, 4, 256)
    q, k, v = _inputs(1, 4, 1, 256, 1024 + 256, seed=3)
    out = G.tree_attention(q, k, v, parents=par, max_depth=8, backend="tcgen05")
    ref = O.tree_attention_batched(_np(q), _np(k), _np(v), parents=par, max_depth=8)
    np.testing.assert_allclose(_np(out), ref, atol=ATOL, rtol=RTOL)


def test_tc_wide_trees_over_many_units():
    """256-node best-first trees on enough (sequence, kv head) units that the
    kernel takes two 128-row M-tiles per CTA (8-word ancestor masks), against
    the CUDA-core kernel."""
    B, Hq, Hkv, N, P = 4, 32, 8, 256, 700
    rng = random.Random(7)
    pars = torch.tensor([best_first_tree(rng, 4, 4, N)[0] for _ in range(B)], device="cuda")
    q, k, v = _inputs(B, Hq, Hkv, N, P + N, seed=7)
    a = G.fused_tree_verify(q, k, v, pars, max_depth=8, backend="tcgen05")
    b = G.fused_tree_verify(q, k, v, pars, max_depth=8, backend="simt")
    torch.testing.assert_close(a.float(), b.float(), atol=ATOL, rtol=RTOL)


def test_auto_picks_tensor_cores_for_64_node_trees():
    q, k, v = _inputs(1, 32, 8, 64, 512)
    par = _trees(1, 64, 0)[0]
    assert G.tree_attention_plan(q, k, v, parents=par)["backend"] == "tcgen05"
    q2, k2, v2 = _inputs(1, 32, 8, 31, 512)
    assert G.tree_attention_plan(q2, k2, v2, parents=_trees(1, 31, 0)[0])["backend"] == "simt"


@pytest.mark.parametrize("grid", [1, 7, 16, 33])
def test_tc_explicit_grid_sizes(grid):
    """num_splits sets the tcgen05 grid: one CTA per pair (16), pairs cut
    between CTAs (7, 33) and a single CTA walking every pair (1)."""
    B, N, P = 2, 64, 700
    pars = torch.tensor(_trees(B, N, seed=grid), device="cuda")
    q, k, v = _inputs(B, 32, 8, N, P + N, seed=grid)
    a = G.fused_tree_verify(q, k, v, pars, max_depth=5, backend="tcgen05", num_splits=grid)
    assert G.tree_attention_plan(q, k, v, parents=pars, backend="tcgen05", num_splits=grid)["splits"] == grid
    b = G.fused_tree_verify(q, k, v, pars, max_depth=5, backend="simt")
    torch.testing.assert_close(a.float(), b.float(), atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("grid,out_dtype", [(100, None), (148, torch.float32)])
def test_tc_many_pieces_per_unit(grid, out_dtype):
    """Grids far above the unit count cut every unit into many pieces (up to
    ten per unit here, odd and even counts): the last piece to finish a warp's
    rows merges them all, output and log-sum-exp, in any output dtype."""
    B, N, P = 1, 64, 2048
    pars = torch.tensor(_trees(B, N, seed=grid), device="cuda")
    q, k, v = _inputs(B, 32, 8, N, P + N, seed=grid)
    plan = G.tree_attention_plan(q, k, v, parents=pars, backend="tcgen05", num_splits=grid, out_dtype=out_dtype)
    assert plan["splits"] == grid and plan["launches"] == 2
    a, la = G.tree_attention(q, k, v, parents=pars, max_depth=5, backend="tcgen05", num_splits=grid,
                             out_dtype=out_dtype, return_lse=True)
    b, lb = G.tree_attention(q, k, v, parents=pars, max_depth=5, backend="simt", out_dtype=out_dtype,
                             return_lse=True)
    assert a.dtype == b.dtype
    torch.testing.assert_close(a.float(), b.float(), atol=ATOL, rtol=RTOL)
    torch.testing.assert_close(la, lb, atol=1e-3, rtol=1e-4)


# ---- units cut between the CTAs of a thread-block cluster (merged in the same launch)

@pytest.mark.parametrize("B,Hq,Hkv,N,P", [
    (1, 32, 8, 64, 2048),    # one sequence: 8 or 16 units, clusters of 8 / 4
    (2, 32, 8, 64, 8192),    # the one-GPU share of an 8-way sequence split
    (1, 8, 2, 100, 1500),    # two query groups per kv head, a partly filled unit
    (1, 4, 4, 256, 900),     # 256-node trees
    (3, 32, 8, 64, 131),     # few tiles per unit: small clusters, one tile per CTA
])
def test_cluster_plan_matches_oracle(B, Hq, Hkv, N, P):
    pars = _trees(B, N, seed=N + P + 1)
    q, k, v = _inputs(B, Hq, Hkv, N, P + N, seed=P + 1)
    par_t = torch.tensor(pars, device="cuda")
    plan = G.tree_attention_plan(q, k, v, parents=par_t, max_depth=5, backend="tcgen05")
    # one launch: the pieces merge inside the kernel, after the cluster barrier
    assert plan["launches"] == 1
    out = G.tree_attention(q, k, v, parents=par_t, max_depth=5, backend="tcgen05")
    if B * Hq * N * (P + N) <= 40_000_000:
        ref = O.tree_attention_batched(_np(q), _np(k), _np(v), parents=np.array(pars), max_depth=5)
        np.testing.assert_allclose(_np(out), ref, atol=ATOL, rtol=RTOL)
    else:  # oracle on sampled (sequence, head) slices
        for b, h in ((0, 0), (B - 1, Hq - 1), (B // 2, Hq // 2 + 1)):
            ref = O.fused_tree_verify(_np(q[b, h]), _np(k[b, h // (Hq // Hkv)]), _np(v[b, h // (Hq // Hkv)]),
                                      pars[b], 5)
            np.testing.assert_allclose(_np(out[b, h]), ref, atol=ATOL, rtol=RTOL)


def test_cluster_lse_fp32_and_head_major_output():
    """The merge writes every output form: fp32 rows, log-sum-exp, and a
    head-major view (a head-sharded layer's output buffer)."""
    B, Hq, Hkv, N, P = 2, 32, 8, 64, 1500
    pars = _trees(B, N, seed=21)
    q, k, v = _inputs(B, Hq, Hkv, N, P + N, seed=21)
    par_t = torch.tensor(pars, device="cuda")
    assert G.tree_attention_plan(q, k, v, parents=par_t, max_depth=5, backend="tcgen05")["launches"] == 1
    out, lse = G.tree_attention(q, k, v, parents=par_t, max_depth=5, backend="tcgen05",
                                out_dtype=torch.float32, return_lse=True)
    _, lse_s = G.tree_attention(q, k, v, parents=par_t, max_depth=5, backend="simt", return_lse=True)
    ref = O.tree_attention_batched(_np(q), _np(k), _np(v), parents=np.array(pars), max_depth=5)
    assert out.dtype == torch.float32
    np.testing.assert_allclose(_np(out), ref, atol=ATOL, rtol=RTOL)
    np.testing.assert_allclose(_np(lse), _np(lse_s), atol=2e-3, rtol=1e-4)
    full = torch.empty(Hq, B, N, 128, device="cuda", dtype=torch.bfloat16)
    hm = full.permute(1, 0, 2, 3)
    G.tree_attention(q, k, v, parents=par_t, max_depth=5, backend="tcgen05", out=hm)
    np.testing.assert_allclose(_np(hm), ref, atol=ATOL, rtol=RTOL)


def test_cluster_row_that_sees_nothing_is_nan():
    """No prefix and a tree-mask row with no visible node: that row is NaN
    with log-sum-exp -inf (softmax over nothing), the others match the oracle."""
    B, Hq, Hkv, N = 1, 8, 8, 200
    par = _trees(1, N, seed=4, depth=6)[0]
    m = G.build_tree_mask(par).clone()
    m[5] = 0
    q, k, v = _inputs(B, Hq, Hkv, N, N, seed=4)
    assert G.tree_attention_plan(q, k, v, m, backend="tcgen05")["launches"] == 1
    out, lse = G.tree_attention(q, k, v, m, backend="tcgen05", return_lse=True)
    o = _np(out)
    assert np.isnan(o[:, :, 5]).all() and np.isneginf(_np(lse)[:, :, 5]).all()
    keep = [i for i in range(N) if i != 5]
    ref = O.tree_attention_batched(_np(q), _np(k), _np(v), mask=_np(m).astype(bool))
    np.testing.assert_allclose(o[:, :, keep], ref[:, :, keep], atol=ATOL, rtol=RTOL)


def test_ragged_sorted_whole_units_match_oracle():
    """A ragged batch with more one-M-tile units than SMs (12 sequences x 8
    kv heads x 2 = 192): whole units ranked by tile count on the device and
    dealt out longest first, two launches (the schedule kernel and the
    attention), no merge kernel; every sequence against the oracle."""
    rng = random.Random(31)
    B, Hq, Hkv, N, D = 12, 32, 8, 64, 128
    Ls = [rng.randint(16, 3000) + N for _ in range(B)]
    cu = np.concatenate([[0], np.cumsum(Ls)]).astype(np.int32)
    pars = _trees(B, N, seed=31)
    g = torch.Generator(device="cuda").manual_seed(31)
    s = 1 / math.sqrt(D)
    q = (torch.randn(B, Hq, N, D, device="cuda", generator=g) * s).bfloat16()
    kp = (torch.randn(int(cu[-1]), Hkv, D, device="cuda", generator=g) * s).bfloat16()
    vp = (torch.randn(int(cu[-1]), Hkv, D, device="cuda", generator=g) * s).bfloat16()
    kw = dict(parents=torch.tensor(pars, device="cuda"), max_depth=5,
              cu_seqlens=torch.from_numpy(cu).cuda(), max_seqlen=max(Ls))
    plan = G.tree_attention_plan(q, kp, vp, **kw, backend="tcgen05")
    assert plan["backend"] == "tcgen05" and plan["launches"] == 2
    out, lse = G.tree_attention(q, kp, vp, **kw, backend="tcgen05", return_lse=True)
    _, lse_s = G.tree_attention(q, kp, vp, **kw, backend="simt", return_lse=True)
    np.testing.assert_allclose(_np(lse), _np(lse_s), atol=2e-3, rtol=1e-4)
    for b in range(B):
        kb = _np(kp[cu[b]:cu[b + 1]]).transpose(1, 0, 2)[None]
        vb = _np(vp[cu[b]:cu[b + 1]]).transpose(1, 0, 2)[None]
        ref = O.tree_attention_batched(_np(q[b:b + 1]), kb, vb, parents=pars[b], max_depth=5)
        np.testing.assert_allclose(_np(out[b:b + 1]), ref, atol=ATOL, rtol=RTOL)
