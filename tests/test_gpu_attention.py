"""Tree attention on the GPU against the oracle.

The first block re-points the reference's own kernel tests
(tests/test_tree_attention_cuda.py:8-20, tests/test_tree_attention_triton.py,
tests/test_fused_tree_verify_triton.py:41-128) at this library, with their
1e-4 tolerance for fp32.  The rest covers what the reference never tested:
prefix, grouped-query heads, batch, bf16 (2e-3 abs / 1e-2 rel against an fp32
oracle on the same bf16-rounded inputs), ragged sequences, split-K."""
from __future__ import annotations

import math
import random

import numpy as np
import pytest
import torch

import projectgorgon_b200 as G
from conftest import load_golden
from oracle import gorgon_oracle as O
from projectgorgon_b200.trees import cartesian_tree, random_tree, reference_random_tree

pytestmark = pytest.mark.gpu
ATT = load_golden("attention")
BF16_ATOL, BF16_RTOL = 2e-3, 1e-2


def _np(t):
    return t.detach().float().cpu().numpy()


# ---------------- reference tests, re-pointed ----------------
@pytest.mark.parametrize("fn", [G.tree_attention_cuda, G.tree_attention_triton])
def test_reference_three_node_case(fn):
    torch.manual_seed(0)
    parents = [-1, 0, 0]
    mask = G.build_tree_mask(parents).to("cuda")
    q = torch.randn(3, 4, device="cuda")
    k = torch.randn(3, 4, device="cuda")
    v = torch.randn(3, 4, device="cuda")
    expected = O.tree_attention(_np(q), _np(k), _np(v), _np(mask) > 0)
    actual = fn(q, k, v, mask)
    assert np.allclose(_np(actual), expected, atol=1e-4, rtol=1e-4)


def _fused_case(parents, dim, max_depth):
    n = len(parents)
    q = torch.randn(n, dim, device="cuda")
    k = torch.randn(n, dim, device="cuda")
    v = torch.randn(n, dim, device="cuda")
    ref = O.tree_attention(_np(q), _np(k), _np(v), O.build_tree_mask(parents))
    got = G.fused_tree_verify(q, k, v, parents, max_depth=max_depth)
    torch.testing.assert_close(got.cpu(), torch.from_numpy(ref), atol=1e-4, rtol=1e-4)


@pytest.mark.parametrize("dim", [32, 64, 128])
def test_fused_chain(dim):
    _fused_case([-1, 0, 1, 2], dim, 4)


@pytest.mark.parametrize("dim", [32, 64, 128])
def test_fused_binary(dim):
    _fused_case([-1, 0, 0, 1, 1], dim, 3)


def test_fused_wide():
    _fused_case([-1, -1, -1, -1, 0, 0, 0, 1, 1, 1, 2, 2, 2, 3, 3, 3], 64, 2)


@pytest.mark.parametrize("n,dim", [(1, 32), (7, 64), (20, 128), (50, 64)])
def test_fused_medusa_like(n, dim):
    random.seed(42)
    parents = [-1]
    for i in range(1, n):
        parents.append(random.randint(0, i - 1))
    _fused_case(parents, dim, n)


def test_fused_tensor_parents():
    parents_list = [-1, 0, 0, 1, 1]
    parents_tensor = torch.tensor(parents_list, dtype=torch.int32, device="cuda")
    q, k, v = (torch.randn(5, 64, device="cuda") for _ in range(3))
    a = G.fused_tree_verify(q, k, v, parents_list, max_depth=3)
    b = G.fused_tree_verify(q, k, v, parents_tensor, max_depth=3)
    torch.testing.assert_close(a, b, atol=1e-6, rtol=1e-6)


def test_fused_single_node():
    _fused_case([-1], 64, 1)


@pytest.mark.parametrize("name", list(ATT["names"]))
def test_golden_attention(name):
    q, k, v, m = (torch.from_numpy(ATT[f"{name}_{x}"]).cuda() for x in ("q", "k", "v", "mask"))
    got = G.tree_attention_triton(q, k, v, m)
    np.testing.assert_allclose(_np(got), ATT[f"{name}_out"], atol=1e-4, rtol=1e-4, equal_nan=True)


def test_max_depth_truncates_like_reference():
    par = reference_random_tree(30, 42)
    q, k, v = (torch.randn(30, 64, device="cuda") for _ in range(3))
    got = G.fused_tree_verify(q, k, v, par, max_depth=2)
    ref = O.fused_tree_verify(_np(q), _np(k), _np(v), par, max_depth=2)
    np.testing.assert_allclose(_np(got), ref, atol=1e-4, rtol=1e-4)


# ---------------- prefix / GQA / batch / bf16 ----------------
def _inputs(B, Hq, Hkv, N, L, D, dtype, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    s = 1.0 / math.sqrt(D)
    q = (torch.randn(B, Hq, N, D, device="cuda", generator=g) * s).to(dtype)
    k = (torch.randn(B, Hkv, L, D, device="cuda", generator=g) * s).to(dtype)
    v = (torch.randn(B, Hkv, L, D, device="cuda", generator=g) * s).to(dtype)
    return q, k, v


def _check(got, ref, dtype):
    if dtype == torch.float32:
        np.testing.assert_allclose(_np(got), ref, atol=1e-4, rtol=1e-4)
    else:
        np.testing.assert_allclose(_np(got), ref, atol=BF16_ATOL, rtol=BF16_RTOL)


def test_c1_shape_fp32_cartesian_tree_prefix_512():
    """fp32, batch 1, 32 heads (kv heads = q heads), d=128, prefix 512,
    31-node Cartesian tree, dense [ones(N,P) | tree mask]."""
    par = cartesian_tree(4, 2, True)
    N, P = len(par), 512
    q, k, v = _inputs(1, 32, 32, N, P + N, 128, torch.float32)
    mask = torch.from_numpy(O.prefix_tree_mask(par, P)).cuda()
    got = G.tree_attention(q, k, v, mask)
    ref = O.tree_attention_batched(_np(q), _np(k), _np(v), mask=mask.cpu().numpy())
    _check(got, ref, torch.float32)
    got2 = G.fused_tree_verify(q, k, v, par, max_depth=len(par))
    _check(got2, ref, torch.float32)


@pytest.mark.parametrize("backend", ["auto", "simt"])
def test_c2_shape_bf16_gqa_parents(backend):
    """bf16, 32 q / 8 kv heads, d=128, prefix 2048, 64-node random tree of
    depth <= 5, mask-free (parents only)."""
    par = random_tree(64, random.Random(0), 5)
    N, P = 64, 2048
    q, k, v = _inputs(1, 32, 8, N, P + N, 128, torch.bfloat16)
    got = G.fused_tree_verify(q, k, v, par, max_depth=5, backend=backend)
    assert got.dtype == torch.bfloat16
    ref = O.tree_attention_batched(_np(q), _np(k), _np(v), parents=par, max_depth=5)
    _check(got, ref, torch.bfloat16)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_batched_per_sequence_trees(dtype):
    B, Hq, Hkv, N, P, D = 3, 8, 2, 24, 300, 64
    pars = [random_tree(N, random.Random(10 + b), 4) for b in range(B)]
    q, k, v = _inputs(B, Hq, Hkv, N, P + N, D, dtype, seed=3)
    got = G.tree_attention(q, k, v, parents=torch.tensor(pars, device="cuda"), max_depth=4)
    ref = O.tree_attention_batched(_np(q), _np(k), _np(v), parents=np.array(pars), max_depth=4)
    _check(got, ref, dtype)


def test_ragged_cu_seqlens():
    """Packed varlen K/V [sum L_b, Hkv, D] with cu_seqlens; each sequence its
    own prefix length and tree."""
    rng = random.Random(4)
    B, Hq, Hkv, N, D = 4, 8, 2, 16, 128
    Ps = [rng.randint(100, 700) for _ in range(B)]
    Ls = [p + N for p in Ps]
    cu = np.concatenate([[0], np.cumsum(Ls)]).astype(np.int32)
    pars = [random_tree(N, random.Random(20 + b), 5) for b in range(B)]
    g = torch.Generator(device="cuda").manual_seed(9)
    s = 1 / math.sqrt(D)
    q = (torch.randn(B, Hq, N, D, device="cuda", generator=g) * s).bfloat16()
    kp = (torch.randn(int(cu[-1]), Hkv, D, device="cuda", generator=g) * s).bfloat16()
    vp = (torch.randn(int(cu[-1]), Hkv, D, device="cuda", generator=g) * s).bfloat16()
    got = G.tree_attention(q, kp, vp, parents=torch.tensor(pars, device="cuda"), max_depth=5,
                           cu_seqlens=torch.from_numpy(cu).cuda(), max_seqlen=max(Ls))
    for b in range(B):
        kb = _np(kp[cu[b]:cu[b + 1]]).transpose(1, 0, 2)[None]
        vb = _np(vp[cu[b]:cu[b + 1]]).transpose(1, 0, 2)[None]
        ref = O.tree_attention_batched(_np(q[b:b + 1]), kb, vb, parents=pars[b], max_depth=5)
        _check(got[b:b + 1], ref, torch.bfloat16)


def test_dense_full_mask_with_masked_prefix_rows():
    B, H, N, P, D = 2, 4, 10, 70, 64
    q, k, v = _inputs(B, H, H, N, P + N, D, torch.float32, seed=5)
    g = torch.Generator().manual_seed(1)
    mask = torch.rand(B, N, P + N, generator=g) > 0.3
    mask[:, :, P:] = torch.from_numpy(O.build_tree_mask(reference_random_tree(N, 1)))
    got = G.tree_attention(q, k, v, mask.cuda())
    ref = O.tree_attention_batched(_np(q), _np(k), _np(v), mask=mask.numpy())
    _check(got, ref, torch.float32)


def test_dense_tree_only_mask_sees_prefix():
    par = reference_random_tree(12, 3)
    N, P = 12, 45
    q, k, v = _inputs(2, 4, 2, N, P + N, 32, torch.bfloat16, seed=6)
    got = G.tree_attention(q, k, v, G.build_tree_mask(par))
    ref = O.tree_attention_batched(_np(q), _np(k), _np(v), parents=par)
    _check(got, ref, torch.bfloat16)


@pytest.mark.parametrize("splits", [1, 3, 17])
def test_split_counts_and_lse(splits):
    par = random_tree(40, random.Random(2), 5)
    N, P = 40, 1000
    q, k, v = _inputs(2, 8, 2, N, P + N, 128, torch.bfloat16, seed=7)
    out, lse = G.tree_attention(q, k, v, parents=par, max_depth=5, num_splits=splits,
                                return_lse=True, backend="simt")
    ref = O.tree_attention_batched(_np(q), _np(k), _np(v), parents=par, max_depth=5)
    _check(out, ref, torch.bfloat16)
    qf, kf = _np(q).astype(np.float64), _np(k).astype(np.float64)
    m = O.prefix_tree_mask(par, P, 5)
    for b in range(2):
        for h in range(8):
            s = qf[b, h] @ kf[b, h // 4].T / math.sqrt(128)
            s = np.where(m, s, -np.inf)
            mx = s.max(-1)
            want = mx + np.log(np.exp(s - mx[:, None]).sum(-1))
            np.testing.assert_allclose(_np(lse[b, h]), want, atol=1e-4, rtol=1e-5)


def test_fp32_output_from_bf16_inputs():
    par = reference_random_tree(9, 0)
    q, k, v = _inputs(1, 4, 4, 9, 9 + 33, 64, torch.bfloat16, seed=8)
    out = G.tree_attention(q, k, v, parents=par, out_dtype=torch.float32)
    assert out.dtype == torch.float32
    ref = O.tree_attention_batched(_np(q), _np(k), _np(v), parents=par)
    np.testing.assert_allclose(_np(out), ref, atol=1e-4, rtol=1e-3)


def test_bad_parent_and_short_sequence_flag_errors():
    G.device_error(clear=True)
    q, k, v = _inputs(1, 2, 2, 4, 10, 32, torch.float32)
    G.fused_tree_verify(q, k, v, torch.tensor([-1, 0, 7, 1], device="cuda"), max_depth=4)
    torch.cuda.synchronize()
    assert G.device_error(clear=True) & 1
