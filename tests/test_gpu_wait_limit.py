"""Failure detection in the tensor-core kernels without a GPU fault: every
wait inside them (on a copy, an MMA, another warp or the other CTA of a
pair) is bounded.  With the bound cut to 1 ns through the C ABI's
gorgon_set_wait_limit_ns, the first wait that is not already satisfied runs
out, as a wait on a flag that nothing sets would; the kernel must then stop,
drain what it issued, free its tensor memory, return and raise bit 4 of the
device error word, leaving the CUDA context usable: the next call with the
normal bound matches the oracle."""
from __future__ import annotations

import math
import random

import numpy as np
import pytest
import torch

import projectgorgon_b200 as G
from oracle import gorgon_oracle as O
from projectgorgon_b200 import _abi
from projectgorgon_b200.trees import random_tree

pytestmark = pytest.mark.gpu


def _case(B, P, seed):
    N, Hq, Hkv, D = 64, 32, 8, 128
    rng = random.Random(seed)
    pars = [random_tree(N, rng, 5) for _ in range(B)]
    g = torch.Generator(device="cuda").manual_seed(seed)
    s = 1.0 / math.sqrt(D)
    q = (torch.randn(B, Hq, N, D, device="cuda", generator=g) * s).bfloat16()
    k = (torch.randn(B, Hkv, P + N, D, device="cuda", generator=g) * s).bfloat16()
    v = (torch.randn(B, Hkv, P + N, D, device="cuda", generator=g) * s).bfloat16()
    return q, k, v, pars


@pytest.mark.parametrize("backend,B,splits", [
    ("tcgen05-cta", 2, None),   # units cut between the CTAs of clusters: every CTA still meets both cluster barriers
    ("tcgen05-cta", 2, 40),     # stream-K pieces and the merge kernel
    ("tcgen05-pair", 16, None),
])
def test_wait_that_runs_out_stops_the_kernel_and_reports_it(backend, B, splits):
    q, k, v, pars = _case(B, 2000, seed=B)
    par_t = torch.tensor(pars, device="cuda")
    kw = {} if splits is None else {"num_splits": splits}
    G.device_error(clear=True)
    prev = _abi.set_wait_limit_ns(1)
    try:
        G.fused_tree_verify(q, k, v, par_t, max_depth=5, backend=backend, **kw)
        torch.cuda.synchronize()
    finally:
        _abi.set_wait_limit_ns(prev)
    assert prev == 2_000_000_000
    assert G.device_error(clear=True) & _abi.ERR_TIMEOUT
    # the context is intact: the same call with the normal bound is right
    out = G.fused_tree_verify(q, k, v, par_t, max_depth=5, backend=backend, **kw)
    torch.cuda.synchronize()
    assert G.device_error(clear=True) == 0
    for b, h in ((0, 0), (B - 1, 31)):
        ref = O.fused_tree_verify(q[b, h].float().cpu().numpy(), k[b, h // 4].float().cpu().numpy(),
                                  v[b, h // 4].float().cpu().numpy(), pars[b], 5)
        np.testing.assert_allclose(out[b, h].float().cpu().numpy(), ref, atol=2e-3, rtol=1e-2)
