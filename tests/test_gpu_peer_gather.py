"""The output gather fused into the tensor-core attention
(``gorgon_tree_attn_gather`` through ``sharding.PeerHeadOutput``): a layer
split by kv head, every rank writing its query heads into every rank's
buffer from the kernel's epilogue over NVLink, with no all-gather call.

One GPU: a group of one is the plain call.  Two GPUs (skipped with fewer):
two processes, one per GPU, exchange buffer handles over a gloo group (no
NCCL on the data path).  The assembled layer on each rank must match the
same rank's own single-GPU attention over all heads, eagerly and in CUDA
graph replays, and the oracle on sampled (sequence, head) slices.  A rank
that never calls makes the other rank's bounded waits run out: the call
raises bit 4 of the device error word instead of hanging, and the CUDA
context stays usable.

Tolerance: bf16 outputs within 2e-3 abs / 1e-2 rel of the fp32 oracle and
of the single-GPU kernel (the per-rank shape may take another plan)."""
from __future__ import annotations

import math
import os
import random
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-3, 1e-2


def _layer(B, Hq, Hkv, N, P, device, seed=0):
    from projectgorgon_b200.trees import random_tree
    g = torch.Generator(device=device).manual_seed(seed)
    s = 1.0 / math.sqrt(128)
    q = (torch.randn(B, Hq, N, 128, device=device, generator=g) * s).bfloat16()
    k = (torch.randn(B, Hkv, P + N, 128, device=device, generator=g) * s).bfloat16()
    v = (torch.randn(B, Hkv, P + N, 128, device=device, generator=g) * s).bfloat16()
    pars = [random_tree(N, random.Random(seed + b), 5) for b in range(B)]
    return q, k, v, pars


def test_group_of_one_is_the_plain_call():
    import projectgorgon_b200 as G
    from projectgorgon_b200 import sharding
    B, Hq, Hkv, N, P = 4, 32, 8, 64, 1000
    q, k, v, pars = _layer(B, Hq, Hkv, N, P, "cuda")
    par_t = torch.tensor(pars, device="cuda", dtype=torch.int32)
    peer = sharding.PeerHeadOutput(B, Hq, Hkv, N, 128, torch.bfloat16, torch.device("cuda", 0), 1, 0)
    try:
        G.fused_tree_verify(q, k, v, par_t, max_depth=5, out=peer.local, peer_group=peer)
        ref = G.fused_tree_verify(q, k, v, par_t, max_depth=5)
        torch.cuda.synchronize()
        assert torch.equal(peer.full, ref)
        assert G.device_error(clear=True) == 0
    finally:
        peer.close()


def test_gather_refuses_an_output_past_the_data_region():
    """The fused gather writes the same offsets in every peer's buffer, so an
    output view that runs into the signal words is refused before anything
    launches (checked here with a two-entry group on one GPU)."""
    import ctypes
    import projectgorgon_b200 as G
    from projectgorgon_b200 import _abi, sharding
    B, Hq, Hkv, N, P = 2, 32, 8, 64, 300
    q, k, v, pars = _layer(B, Hq, Hkv, N, P, "cuda")
    par_t = torch.tensor(pars, device="cuda", dtype=torch.int32)
    peer = sharding.PeerHeadOutput(B, Hq, Hkv, N, 128, torch.bfloat16, torch.device("cuda", 0), 1, 0)
    try:
        own = peer.full_head_major.data_ptr()
        bases = (ctypes.c_void_p * _abi.MAX_PEERS)(own, own)

        class _TwoRanks:
            group = _abi.PeerGroup(2, 0, bases, peer.signal_offset)

            def group_ref(self):
                return ctypes.byref(self.group)

        full = peer.full_head_major
        shifted = full.as_strided(full.shape, full.stride(), full.storage_offset() + 8).permute(1, 0, 2, 3)
        with pytest.raises(RuntimeError, match="data region"):
            G.fused_tree_verify(q, k, v, par_t, max_depth=5, out=shifted, peer_group=_TwoRanks())
        torch.cuda.synchronize()
        assert G.device_error(clear=True) == 0
    finally:
        peer.close()


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _check_gather(G, O, dist, peer, qa, ka, va, ql, kl, vl, pars, par_t):
    """Eager calls, then one captured call replayed: the assembled layer
    against this GPU's own attention over all heads and the oracle."""
    B, Hq = qa.shape[0], qa.shape[1]
    ref = G.fused_tree_verify(qa, ka, va, par_t, max_depth=5)
    for _ in range(3):
        peer.full_head_major.zero_()
        dist.barrier()
        G.fused_tree_verify(ql, kl, vl, par_t, max_depth=5, out=peer.local, peer_group=peer)
        torch.cuda.synchronize()
        torch.testing.assert_close(peer.full.float(), ref.float(), atol=ATOL, rtol=RTOL)
    # captured once, replayed: the signal counters advance on the device
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        G.fused_tree_verify(ql, kl, vl, par_t, max_depth=5, out=peer.local, peer_group=peer)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        G.fused_tree_verify(ql, kl, vl, par_t, max_depth=5, out=peer.local, peer_group=peer)
    for _ in range(3):
        peer.full_head_major.zero_()
        torch.cuda.synchronize()
        dist.barrier()
        graph.replay()
        torch.cuda.synchronize()
        torch.testing.assert_close(peer.full.float(), ref.float(), atol=ATOL, rtol=RTOL)
    del graph
    for b, h in ((0, 0), (B - 1, Hq - 1), (1, Hq // 2 + 3)):
        o = O.fused_tree_verify(qa[b, h].float().cpu().numpy(), ka[b, h // 4].float().cpu().numpy(),
                                va[b, h // 4].float().cpu().numpy(), pars[b], 5)
        np.testing.assert_allclose(peer.full[b, h].float().cpu().numpy(), o, atol=ATOL, rtol=RTOL)
    assert G.device_error(clear=True) == 0


def _rank_main(rank, world, port, mode, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        import datetime
        import torch.distributed as dist
        import projectgorgon_b200 as G
        from oracle import gorgon_oracle as O
        from projectgorgon_b200 import _abi, sharding
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        msg = "ok"
        # a cluster plan (16 units per rank) and a whole-unit plan (128 units per rank)
        shapes = [(4, 1500), (32, 300)] if mode == "gather" else [(4, 1500)]
        for B, P in shapes:
            Hq, Hkv, N = 32, 8, 64
            qa, ka, va, pars = _layer(B, Hq, Hkv, N, P, dev)     # the whole layer, same on every rank
            par_t = torch.tensor(pars, device=dev, dtype=torch.int32)
            (h0, h1), (q0, q1) = sharding.shard_heads(Hkv, Hq, world, rank)
            ql, kl, vl = qa[:, q0:q1].contiguous(), ka[:, h0:h1].contiguous(), va[:, h0:h1].contiguous()
            peer = sharding.PeerHeadOutput(B, Hq, Hkv, N, 128, torch.bfloat16, dev, world, rank)
            if mode == "gather":
                _check_gather(G, O, dist, peer, qa, ka, va, ql, kl, vl, pars, par_t)
            else:  # "absent": rank 1 never calls, rank 0's waits run out
                if rank == 0:
                    prev = _abi.set_wait_limit_ns(100_000_000)
                    try:
                        G.fused_tree_verify(ql, kl, vl, par_t, max_depth=5, out=peer.local, peer_group=peer)
                        torch.cuda.synchronize()
                    finally:
                        _abi.set_wait_limit_ns(prev)
                    err = G.device_error(clear=True)
                    assert err & _abi.ERR_TIMEOUT, err
                    # the context is intact: a plain call on this GPU is right
                    out = G.fused_tree_verify(ql, kl, vl, par_t, max_depth=5)
                    torch.cuda.synchronize()
                    ref = O.fused_tree_verify(ql[0, 0].float().cpu().numpy(), kl[0, 0].float().cpu().numpy(),
                                              vl[0, 0].float().cpu().numpy(), pars[0], 5)
                    np.testing.assert_allclose(out[0, 0].float().cpu().numpy(), ref, atol=ATOL, rtol=RTOL)
                    assert G.device_error(clear=True) == 0
                dist.barrier()
            peer.close()
        dist.destroy_process_group()
        q.put((rank, msg))
    except BaseException as exc:  # pragma: no cover - reported to the parent
        q.put((rank, repr(exc)))


def _run_two(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, msg in results:
        assert msg == "ok", (rank, msg)
    assert all(p.exitcode == 0 for p in procs)


two_gpus = pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")


@two_gpus
def test_two_gpus_gather_matches_the_whole_layer():
    _run_two("gather")


@two_gpus
def test_peer_that_never_calls_makes_the_waits_run_out():
    _run_two("absent")
