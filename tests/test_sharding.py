"""Multi-rank host logic of the verify path, run as two gloo ranks on CPU:
sequence and kv-head sharding, the slowest-rank timing reduction and the
output gathers."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from projectgorgon_b200 import sharding


def test_shard_range_covers_items_once():
    for n in (0, 1, 7, 16, 33):
        for world in (1, 2, 3, 8):
            spans = [sharding.shard_range(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[r][1] == spans[r + 1][0] for r in range(world - 1))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1


def test_shard_by_weight_balances_ragged_rows():
    import random
    rng = random.Random(0)
    w = [rng.randint(1024, 8192) + 64 for _ in range(64)]
    for world in (1, 2, 4, 8):
        spans = [sharding.shard_by_weight(w, world, r) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == len(w)
        assert all(spans[r][1] == spans[r + 1][0] for r in range(world - 1))
        loads = [sum(w[a:b]) for a, b in spans]
        assert max(loads) - sum(w) / world <= max(w)


def test_shard_rejects_bad_rank():
    with pytest.raises(ValueError):
        sharding.shard_range(4, 2, 2)


def test_shard_heads_keeps_gqa_groups_together():
    for world in (1, 2, 4, 8):
        spans = [sharding.shard_heads(8, 32, world, r) for r in range(world)]
        assert spans[0][0][0] == 0 and spans[-1][0][1] == 8 and spans[-1][1][1] == 32
        for (h0, h1), (q0, q1) in spans:
            assert q0 == 4 * h0 and q1 == 4 * h1 and h1 - h0 == 8 // world
    with pytest.raises(ValueError):
        sharding.shard_heads(8, 32, 3, 0)


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    try:
        env = sharding.dist_env()
        sharding.init(env, "gloo", timeout_s=60)
        # slowest rank's time is the job's time; the job's bytes are every rank's
        t = sharding.max_over_ranks(1.5 + rank)
        total = sharding.sum_over_ranks(10 + rank)
        # each rank holds its own sequences' outputs; the gather restores the batch
        # order, also when the shards differ in length (7 sequences: 3 and 4)
        ok = total == 21.0
        for B in (6, 7):
            a, b = sharding.shard_range(B, world, rank)
            full = torch.arange(B * 4, dtype=torch.float32).view(B, 4)
            ok = ok and bool(torch.equal(sharding.gather_batch(full[a:b].clone()), full))
        # each rank holds the outputs of its query heads; the gather restores [B, Hq, N, D]
        o = torch.arange(3 * 8 * 5 * 2, dtype=torch.float32).view(3, 8, 5, 2)
        _, (q0, q1) = sharding.shard_heads(4, 8, world, rank)
        ok = ok and bool(torch.equal(sharding.gather_heads(o[:, q0:q1].clone()), o))
        # head-major buffer: the rank writes its slice in place, the gather fills the rest
        hm, local = sharding.head_sharded_output(3, 8, 5, 2, torch.float32, torch.device("cpu"), world, rank)
        assert local.shape == (3, 4, 5, 2)
        local.copy_(o[:, q0:q1])
        ok = ok and bool(torch.equal(sharding.gather_heads_inplace(hm), o))
        # the asynchronous form: the view is complete once the work is waited on
        hm2, local2 = sharding.head_sharded_output(3, 8, 5, 2, torch.float32, torch.device("cpu"), world, rank)
        local2.copy_(o[:, q0:q1])
        view, work = sharding.gather_heads_inplace(hm2, async_op=True)
        work.wait()
        ok = ok and bool(torch.equal(view, o))
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
        q.put((rank, t, ok))
    except Exception as exc:  # pragma: no cover - reported to the parent
        q.put((rank, None, repr(exc)))


def test_two_gloo_ranks_time_and_gather():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs)
    for rank, t, ok in results:
        assert t == 2.5, (rank, t, ok)
        assert ok is True, (rank, ok)
