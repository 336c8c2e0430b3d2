"""The allocation-free verifier entry point, gorgon_verify_noalloc.

It exists for callers that cannot call cudaMalloc -- hosts that only receive
the buffers an owning framework hands them, or a decode step that must not
add a synchronising allocation -- so it keeps its scratch (one counter per
sequence) in a fixed array inside the library.  These tests call it through
the C ABI and compare it with gorgon_verify, which takes a caller workspace,
on two calls in a row (the second call sees the first call's leftover
counters and must clear them).  This file is collected last on purpose.
"""
from __future__ import annotations

import ctypes
import random

import pytest
import torch

from projectgorgon_b200 import _abi
from projectgorgon_b200.trees import random_tree


def _params(logits, draft, parents, outs, prompt_len=1):
    B, R, V = logits.shape
    p = _abi.VerifyParams()
    p.dtype = _abi.BF16 if logits.dtype == torch.bfloat16 else _abi.F32
    p.logits, p.logits_stride_b, p.logits_stride_r = logits.data_ptr(), logits.stride(0), logits.stride(1)
    p.batch, p.rows, p.vocab, p.n, p.prompt_len = B, R, V, draft.shape[1], prompt_len
    p.draft, p.draft_stride_b = draft.data_ptr(), draft.stride(0)
    p.parents, p.parents_stride_b = parents.data_ptr(), parents.stride(0)
    p.pred, p.accepted_len, p.path = outs["pred"].data_ptr(), outs["len"].data_ptr(), outs["path"].data_ptr()
    p.bonus, p.best_node, p.hidden_row = (outs["bonus"].data_ptr(), outs["best"].data_ptr(),
                                          outs["hidden"].data_ptr())
    return p


def _outs(B, n):
    i32 = dict(dtype=torch.int32, device="cuda")
    return {"pred": torch.full((B, n + 1), -7, **i32), "len": torch.full((B,), -7, **i32),
            "path": torch.full((B, n), -7, **i32), "bonus": torch.full((B,), -7, **i32),
            "best": torch.full((B,), -7, **i32), "hidden": torch.full((B,), -7, **i32)}


@pytest.mark.gpu
def test_noalloc_verifier_matches_workspace_verifier_twice():
    B, n, V = 8, 64, 32000
    rng = random.Random(17)
    g = torch.Generator(device="cuda").manual_seed(17)
    logits = (torch.randn(B, n + 1, V, device="cuda", generator=g) * 2.0).bfloat16()
    pred = logits.float().argmax(-1).cpu()
    parents = torch.tensor([random_tree(n, rng, 5) for _ in range(B)], dtype=torch.int32, device="cuda")
    draft = torch.randint(0, V, (B, n), generator=g, device="cuda", dtype=torch.int32)
    par_h = parents.cpu()
    for b in range(B):
        for t in range(n):
            if rng.random() < 0.6:
                p = int(par_h[b, t])
                draft[b, t] = int(pred[b, 0 if p < 0 else p + 1])
    lib = _abi.lib()
    stream = torch.cuda.current_stream().cuda_stream

    want = _outs(B, n)
    pw = _params(logits, draft, parents, want)
    nbytes = lib.gorgon_verify_workspace_size(pw)
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    _abi.check(lib.gorgon_verify(pw, ws.data_ptr(), nbytes, stream), "gorgon_verify")

    for call in range(2):
        got = _outs(B, n)
        _abi.check(lib.gorgon_verify_noalloc(_params(logits, draft, parents, got), stream),
                   "gorgon_verify_noalloc")
        torch.cuda.synchronize()
        for key in want:
            assert torch.equal(got[key], want[key]), (call, key)
    assert int(want["len"].max()) > 0  # the comparison covers accepted paths


def test_noalloc_rejects_batches_beyond_its_fixed_scratch():
    p = _abi.VerifyParams()
    p.dtype, p.batch, p.rows, p.vocab, p.n, p.prompt_len = _abi.BF16, 4097, 2, 10, 1, 1
    rc = _abi.lib().gorgon_verify_noalloc(ctypes.byref(p), None)
    assert rc == _abi.GORGON_ERR_UNSUPPORTED
    assert "4096" in _abi.lib().gorgon_last_error().decode()
