"""Tree-verification benchmark: tree attention over [prefix | tree] on B200.

One step is one tree-verify attention layer over a batch of sequences, run
through the public operator ``fused_tree_verify`` (mask-free, parents only).
The default workload is the Llama-3-8B layer shape: batch 16, 32 query / 8
key-value heads, head_dim 128, prefix 8192, a 64-node random tree per
sequence (depth <= 5), bf16.

Prints one JSON line (rank 0).  ``value`` is algorithmic HBM GB/s of the
whole job (K and V of every sequence read once, Q read once, output written
once, parents read once) with inputs resident in HBM; ``e2e`` is the same
metric with each step's new inputs (Q, the tree's K/V rows, parents) copied
from pinned host memory and the output copied back inside the timed region,
with the time each stage takes on its own stream.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
    python bench.py --impl reference ...   # the reference's attention on the host cores

Multi-GPU (torchrun, one rank per GPU): by default the workload's batch is
split by sequence over the ranks (strong scaling: the same layer on more
GPUs, no collective on the data path); ``--shard weak`` gives every rank a
batch of its own, ``--shard heads`` splits one layer by kv head, the output
gathered by the attention kernel itself over NVLink (``--gather nccl``: an
NCCL all-gather after it).  The timing is the max over ranks.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import random
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import projectgorgon_b200 as G  # noqa: E402
from projectgorgon_b200 import sharding  # noqa: E402
from projectgorgon_b200.trees import best_first_tree, cartesian_tree, random_tree  # noqa: E402

# Per-launch DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of the
# dominant kernel from the ncu captures summarised under profiles/, keyed by
# (workload, backend).  None until a capture exists.
NCU_TRAFFIC_BYTES = {
    # profiles/attn_tc_kernel_verify-b16-p8192-n64.md: 549.566 MB read + 3.622 MB written
    ("verify-b16-p8192-n64", "tcgen05"): 553188096,
    # profiles/attn_tc_kernel_verify-b1-p2048-n64.md (cluster plan): 9.296 MB read, 0 written
    ("verify-b1-p2048-n64", "tcgen05"): 9295616,
    # profiles/verify_kernel_verifier-b32-n64-v128256.md: 570.646 MB read + 4.049 MB written
    ("verifier-b32-n64-v128256", "verify_kernel"): 574694912,
    # profiles/kv_trim_warp_kernel_kvtrim-b32-l32-p4096.md: the 4-layer capture (1.389 MB read,
    # 0 written) scaled by 8 to 32 layers
    ("kvtrim-b32-l32-p4096", "kv_trim_kernel"): 11108352,
    # profiles/cand_segment_kernel_candidates-b32-h4-v128256.md: 32.893 MB read, 0 written
    ("candidates-b32-h4-v128256", "cand_segment_kernel"): 32893440,
    # profiles/attn_tc_kernel_wide-b8-p32k-n256.md: 1100.020 MB read + 16.812 MB written
    ("wide-b8-p32k-n256", "tcgen05"): 1116831744,
    # profiles/head_segment_kernel_medusa-heads-b1-h4-d4096-v128256.md: the one-head capture
    # (1050.718 MB read + 3.665 MB written) and, scaled by the head count, the four-head workload
    ("medusa-heads-b1-h1-d4096-v128256", "head_segment_kernel"): 1054383104,
    ("medusa-heads-b1-h4-d4096-v128256", "head_segment_kernel"): 4217532416,
}

WORKLOADS = {
    "verify-b16-p8192-n64": dict(B=16, Hq=32, Hkv=8, D=128, P=8192, N=64, dtype="bf16",
                                 tree="random", max_depth=5),
    "verify-b1-p2048-n64": dict(B=1, Hq=32, Hkv=8, D=128, P=2048, N=64, dtype="bf16",
                                tree="random", max_depth=5),
    "ref-fp32-b1-p512-n31": dict(B=1, Hq=32, Hkv=32, D=128, P=512, N=31, dtype="fp32",
                                 tree="cartesian", max_depth=31),
    "ragged-b16-p1k-8k-n64": dict(B=16, Hq=32, Hkv=8, D=128, P=(1024, 8192), N=64, dtype="bf16",
                                  tree="random", max_depth=5),
    # one layer of the 32-layer verify tail: 32 sequences over a 4096-token prefix
    "verify-b32-p4096-n64": dict(B=32, Hq=32, Hkv=8, D=128, P=4096, N=64, dtype="bf16",
                                 tree="random", max_depth=5),
    # 256-node best-first trees (top-4 over 4 levels) over a 32k prefix: the
    # tensor-bound shape (arithmetic intensity ~1000 flop/byte)
    "wide-b8-p32k-n256": dict(B=8, Hq=32, Hkv=8, D=128, P=32768, N=256, dtype="bf16",
                              tree="best_first", max_depth=8, bound="tensor"),
    # the fused verifier over one decode step's logits (65 rows: the root's
    # row plus one per node) of a 128256-token vocabulary
    "verifier-b32-n64-v128256": dict(kind="verify", B=32, N=64, V=128256, dtype="bf16", max_depth=5),
    # trim-on-reject of the accepted path (<= 6 rows) in all 32 layers of a
    # [32, 8, 4160, 128] bf16 K and V cache
    "kvtrim-b32-l32-p4096": dict(kind="trim", B=32, layers=32, Hkv=8, D=128, P=4096, N=64, dtype="bf16",
                                 max_depth=5),
    # the same trim over 4 layers (2.2 GB of cache): small enough for a
    # multi-pass profiler capture; its traffic scales with the layer count
    "kvtrim-b32-l4-p4096": dict(kind="trim", B=32, layers=4, Hkv=8, D=128, P=4096, N=64, dtype="bf16",
                                max_depth=5),
    # candidate trees from 4 Medusa heads over a 128256-token vocabulary:
    # per-head top-4, softmax and entropy, then a 64-node budgeted tree
    "candidates-b32-h4-v128256": dict(kind="cand", B=32, heads=4, V=128256, top_k=4, max_candidates=64,
                                      dtype="bf16"),
    # the same trees straight from 4 Medusa heads' last Linear (Llama-3-8B
    # width: 4096 x 128256 bf16 per head, 4.2 GB of weights), one sequence
    "medusa-heads-b1-h4-d4096-v128256": dict(kind="heads", B=1, heads=4, H=4096, V=128256, top_k=4,
                                             max_candidates=64, dtype="bf16"),
    # one such head (1.05 GB of weights): small enough for a multi-pass
    # profiler capture; its traffic scales with the head count
    "medusa-heads-b1-h1-d4096-v128256": dict(kind="heads", B=1, heads=1, H=4096, V=128256, top_k=4,
                                             max_candidates=64, dtype="bf16"),
}
DEFAULT_WORKLOAD = "verify-b16-p8192-n64"
L2_FLUSH_BELOW = 256e6  # bytes per step under which a workload flushes L2 between steps
TORCH_DT = {"bf16": torch.bfloat16, "fp32": torch.float32}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def make_tree(cfg: dict, rng: random.Random):
    """The parents[] of one sequence's candidate tree."""
    if cfg["tree"] == "random":
        return random_tree(cfg["N"], rng, cfg["max_depth"])
    if cfg["tree"] == "best_first":
        return best_first_tree(rng, 4, 4, cfg["N"])[0]
    return cartesian_tree(4, 2, True)


def attn_sequences(cfg: dict, first_seq: int, count: int):
    """(prefix lengths, parents) of global sequences first_seq .. first_seq +
    count - 1.  Sequence j's prefix and tree come from a generator seeded by
    j alone, so any split of the batch over ranks (or the host-side
    reference) sees the same job."""
    prefixes, parents = [], []
    for j in range(first_seq, first_seq + count):
        r = random.Random(1_000_003 + j)
        prefixes.append(r.randint(*cfg["P"]) if isinstance(cfg["P"], tuple) else cfg["P"])
        parents.append(make_tree(cfg, r))
    return prefixes, parents


def attn_bytes(cfg: dict, prefixes) -> int:
    """Algorithmic HBM bytes of the attention over these sequences: K and V of
    every kv head read once over P + N rows, Q read once, the output written
    once, parents (and cu_seqlens for a ragged batch) read once."""
    B, Hq, Hkv, D, N = len(prefixes), cfg["Hq"], cfg["Hkv"], cfg["D"], cfg["N"]
    esz = 2 if cfg["dtype"] == "bf16" else 4
    kv_rows = sum(p + N for p in prefixes)
    return (2 * kv_rows * Hkv * D * esz + 2 * B * Hq * N * D * esz + B * N * 4
            + ((B + 1) * 4 if isinstance(cfg["P"], tuple) else 0))


def attn_flops(cfg: dict, prefixes) -> int:
    """Dense-equivalent FLOPs: 4 * Hq * N * D per key/value row (Q.K^T and P.V)."""
    return 4 * cfg["Hq"] * cfg["N"] * cfg["D"] * sum(p + cfg["N"] for p in prefixes)


def seq_shard(name: str, world: int, rank: int, mode: str):
    """(first sequence, sequence count) of `rank`.  ``strong``: the workload's
    fixed batch split over the ranks (contiguous runs; a ragged batch is cut
    by key/value rows so every rank streams about the same bytes); ``weak``:
    every rank takes a whole batch of its own."""
    cfg = WORKLOADS[name]
    B = cfg["B"]
    if mode == "weak" or world == 1:
        return rank * B if mode == "weak" else 0, B
    if B < world:
        raise SystemExit(f"{name}: {B} sequences cannot be split over {world} ranks (use --shard weak)")
    if cfg.get("kind", "attn") == "attn" and isinstance(cfg["P"], tuple):
        prefixes, _ = attn_sequences(cfg, 0, B)
        s, e = sharding.shard_by_weight([p + cfg["N"] for p in prefixes], world, rank)
    else:
        s, e = sharding.shard_range(B, world, rank)
    return s, e - s


def attn_config(name: str, world: int, mode: str, gather: str = "fused") -> dict:
    """The `config` of an attention workload's JSON line: the same dict for
    this build's arm and the reference arm (it needs no GPU)."""
    cfg = WORKLOADS[name]
    ragged = isinstance(cfg["P"], tuple)
    B = cfg["B"]
    if mode in ("weak", "heads") or world == 1:
        per_gpu = [B] * world
        local_bytes = attn_bytes(cfg, attn_sequences(cfg, 0, B)[0]) // (world if mode == "heads" else 1)
    else:
        per_gpu = [seq_shard(name, world, r, mode)[1] for r in range(world)]
        s0, n0 = seq_shard(name, world, 0, mode)
        local_bytes = attn_bytes(cfg, attn_sequences(cfg, s0, n0)[0])
    if world == 1:
        par = "single GPU"
    elif mode == "weak":
        par = f"sequence-sharded x{world}, weak scaling: {B} sequences per GPU, {B * world} in all"
    elif mode == "heads":
        how = ("the output gather fused into the attention (NVLink stores to every GPU's buffer)"
               if gather == "fused" else "one NCCL all-gather of the output")
        par = f"kv-head-sharded x{world}, strong scaling: {cfg['Hkv'] // world} of {cfg['Hkv']} kv heads per GPU, {how}"
    else:
        par = (f"sequence-sharded x{world}, strong scaling: the batch of {B} sequences split "
               f"{'/'.join(str(n) for n in per_gpu)} over the GPUs, no collective on the data path")
    return {
        "workload": name, "batch": B * world if mode == "weak" else B,
        "batch_per_gpu": per_gpu[0] if len(set(per_gpu)) == 1 else per_gpu,
        "heads_q": cfg["Hq"], "heads_kv": cfg["Hkv"], "head_dim": cfg["D"],
        "prefix": list(cfg["P"]) if ragged else cfg["P"], "tree_nodes": cfg["N"], "tree": cfg["tree"],
        "max_depth": cfg["max_depth"], "mask": "parents (mask-free)", "parallelism": par,
        "l2": ("L2 flushed before every step (a 256 MB write outside the step's events)"
               if local_bytes < L2_FLUSH_BELOW else
               f"inputs larger than L2 ({local_bytes / 1e6:.0f} MB per step per GPU)"),
    }


# --------------------------------------------------------------------------
# workload construction
# --------------------------------------------------------------------------
class Workload:
    """Seeded synthetic inputs of one workload, resident on `dev`.

    Sequence j of this rank is global sequence first_seq + j, and everything
    about it (prefix length, tree, q/k/v) comes from generators seeded by that
    global index, so the union of all ranks' shards is one well-defined job
    whatever the number of ranks."""

    def __init__(self, name: str, dev: torch.device, first_seq: int = 0, batch: int = None):
        cfg = WORKLOADS[name]
        self.name, self.cfg, self.dev = name, cfg, dev
        B = cfg["B"] if batch is None else batch
        Hq, Hkv, D, N = cfg["Hq"], cfg["Hkv"], cfg["D"], cfg["N"]
        self.B, self.first_seq = B, first_seq
        self.ragged = isinstance(cfg["P"], tuple)
        self.prefixes, self.parents = attn_sequences(cfg, first_seq, B)
        self.max_depth = cfg["max_depth"]
        dt = TORCH_DT[cfg["dtype"]]
        self.dtype = dt
        s = 1.0 / math.sqrt(D)
        gens = [torch.Generator(device=dev).manual_seed(first_seq + j) for j in range(B)]
        self.q = torch.empty(B, Hq, N, D, device=dev, dtype=dt)
        for j in range(B):
            self.q[j] = (torch.randn(Hq, N, D, device=dev, generator=gens[j]) * s).to(dt)
        lens = [p + N for p in self.prefixes]
        if self.ragged:
            self.cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32, device=dev)
            total = int(sum(lens))
            self.k = torch.empty(total, Hkv, D, device=dev, dtype=dt)
            self.v = torch.empty(total, Hkv, D, device=dev, dtype=dt)
            off = 0
            for j, L in enumerate(lens):
                self.k[off:off + L] = (torch.randn(L, Hkv, D, device=dev, generator=gens[j]) * s).to(dt)
                self.v[off:off + L] = (torch.randn(L, Hkv, D, device=dev, generator=gens[j]) * s).to(dt)
                off += L
            self.max_seqlen = max(lens)
        else:
            L = lens[0]
            self.cu = None
            self.k = torch.empty(B, Hkv, L, D, device=dev, dtype=dt)
            self.v = torch.empty(B, Hkv, L, D, device=dev, dtype=dt)
            for j in range(B):  # per-sequence fill keeps the fp32 temporary small
                self.k[j] = (torch.randn(Hkv, L, D, device=dev, generator=gens[j]) * s).to(dt)
                self.v[j] = (torch.randn(Hkv, L, D, device=dev, generator=gens[j]) * s).to(dt)
            self.max_seqlen = L
        self.par_t = torch.tensor(self.parents, dtype=torch.int32, device=dev)
        self.bytes = attn_bytes(cfg, self.prefixes)
        self.flops = attn_flops(cfg, self.prefixes)
        self.tokens = B * N
        # a layer that fits in L2 (126 MB) twice over is timed from a flushed L2
        self.flush_l2 = self.bytes < L2_FLUSH_BELOW

    def kwargs(self):
        kw = dict(parents=self.par_t, max_depth=self.max_depth)
        if self.ragged:
            kw.update(cu_seqlens=self.cu, max_seqlen=self.max_seqlen)
        return kw

    def step(self):
        return G.fused_tree_verify(self.q, self.k, self.v, **self.kwargs())

    def plan(self):
        return G.tree_attention_plan(self.q, self.k, self.v, **self.kwargs())

    metric = "tree-verify HBM GB/s (algorithmic bytes / step time)"
    data = "synthetic (seeded N(0,1)/sqrt(128) q/k/v, random trees)"

    @property
    def bound(self):
        return self.cfg.get("bound", "hbm")

    mode = "strong"
    graphable = True  # one step is one stream-ordered public call

    def config(self, world: int, plan: dict) -> dict:
        return attn_config(self.name, world, self.mode, getattr(self, "gather", "fused"))

    def extra(self, world: int, ms_step: float) -> dict:
        return {"us_per_layer": round(ms_step * 1e3, 2),
                "tokens_verified_per_s": round(self.job_tokens(world) / (ms_step * 1e-3), 1)}

    def job_tokens(self, world: int) -> int:
        """Tree tokens verified per step by all ranks together."""
        return self.cfg["B"] * self.cfg["N"] * (world if self.mode == "weak" else 1)

    def e2e(self, steps: int, warmup: int, world: int):
        ms, h2d, d2h, parts = time_e2e(self, steps, warmup, world)
        return ms, h2d, d2h, ("prefix K/V cache resident in HBM; per step the tree's Q, K/V rows and "
                              "parents are copied in and the output copied out, pipelined: step i + 1's "
                              "copy-in and step i - 1's copy-out overlap step i's compute; the *_ms parts "
                              "are each stage's mean duration on its own stream"), parts

    def cpu_baseline(self, budget_s: float):
        return cpu_baseline(self, budget_s=budget_s)


class HeadShardWorkload(Workload):
    """One layer split by kv head over the ranks (``--shard heads``, strong
    scaling): rank r keeps the K/V cache of its Hkv / world kv heads and the
    query heads that read them, computes their outputs, and an NCCL
    all-gather assembles the layer's output [B, Hq, N, D] on every rank.  A
    step is the local attention plus the gather; the attention alone is timed
    beside it (``kernel_only_us``).  Trees and prefixes come from the
    per-sequence seeds, each head's Q, K and V from a (sequence, head) seed,
    so the job is the same for every number of ranks."""

    scaling = "strong"

    def __init__(self, name: str, dev: torch.device, rank: int, world: int, chunks: int = 1,
                 gather: str = "fused"):
        cfg = WORKLOADS[name]
        if isinstance(cfg["P"], tuple):
            raise SystemExit("--shard heads needs a workload with one prefix length")
        if cfg["B"] % chunks:
            raise SystemExit(f"--head-chunks {chunks} does not divide the batch of {cfg['B']}")
        if gather == "fused" and chunks != 1:
            raise SystemExit("--head-chunks applies to --gather nccl")
        self.chunks, self.gather = chunks, gather
        self.name, self.cfg, self.dev = name, cfg, dev
        B, Hq, Hkv, D, N, P = cfg["B"], cfg["Hq"], cfg["Hkv"], cfg["D"], cfg["N"], cfg["P"]
        (h0, h1), (q0, q1) = sharding.shard_heads(Hkv, Hq, world, rank)
        self.world, self.ragged, self.cu = world, False, None
        rngs = [random.Random(1_000_003 + j) for j in range(B)]
        self.prefixes = [P] * B
        self.parents = [make_tree(cfg, r) for r in rngs]
        self.max_depth = cfg["max_depth"]
        dt = TORCH_DT[cfg["dtype"]]
        self.dtype = dt
        s = 1.0 / math.sqrt(D)
        L = P + N
        self.max_seqlen = L
        self.q = torch.empty(B, q1 - q0, N, D, device=dev, dtype=dt)
        self.k = torch.empty(B, h1 - h0, L, D, device=dev, dtype=dt)
        self.v = torch.empty(B, h1 - h0, L, D, device=dev, dtype=dt)
        for j in range(B):
            for qh in range(q0, q1):
                g = torch.Generator(device=dev).manual_seed(5_000_000 + j * Hq + qh)
                self.q[j, qh - q0] = (torch.randn(N, D, device=dev, generator=g) * s).to(dt)
            for h in range(h0, h1):
                g = torch.Generator(device=dev).manual_seed(6_000_000 + j * Hkv + h)
                self.k[j, h - h0] = (torch.randn(L, D, device=dev, generator=g) * s).to(dt)
                self.v[j, h - h0] = (torch.randn(L, D, device=dev, generator=g) * s).to(dt)
        self.par_t = torch.tensor(self.parents, dtype=torch.int32, device=dev)
        # the layer output, head-major per batch chunk: this rank's heads are
        # one contiguous piece of each chunk's buffer, which the attention
        # writes and the in-place all-gather sends; chunk c's gather runs on
        # NCCL's stream while chunk c + 1's attention computes
        self.peers = []
        if gather == "fused":
            # the gather fused into the attention: every rank's heads go
            # straight into every rank's buffer over NVLink (two buffers, so
            # that an end-to-end step's copy-out overlaps the next step)
            self.peers = [sharding.PeerHeadOutput(B, Hq, Hkv, N, D, dt, dev, world, rank) for _ in range(2)]
            self.full, self.local = self.peers[0].full_head_major, self.peers[0].local
            self.fulls, self.locals = [self.full], [self.local]
            self.graphable = True  # no collective call in the step
        else:
            Bc = B // chunks
            bufs = [sharding.head_sharded_output(Bc, Hq, N, D, dt, dev, world, rank) for _ in range(chunks)]
            self.fulls = [f for f, _ in bufs]
            self.locals = [l for _, l in bufs]
            self.full, self.local = bufs[0]
        self.out = torch.empty(B, Hq, N, D, device=dev, dtype=dt)  # shape only (the e2e copy-out buffer)
        esz = torch.tensor([], dtype=dt).element_size()
        # this rank's share: its K/V, Q and output slice, and the parents
        self.bytes = 2 * B * (h1 - h0) * L * D * esz + 2 * B * (q1 - q0) * N * D * esz + B * N * 4
        self.flops = 4 * (q1 - q0) * N * D * B * L
        self.tokens = B * N
        self.kernel_events = []

    def step(self):
        st = torch.cuda.current_stream(self.dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if self.gather == "fused":
            peer = self.peers[0]
            return G.fused_tree_verify(self.q, self.k, self.v, out=peer.local, peer_group=peer, **self.kwargs())
        if self.chunks == 1:
            e0.record(st)
            G.fused_tree_verify(self.q, self.k, self.v, out=self.local, **self.kwargs())
            e1.record(st)
            self.kernel_events.append((e0, e1))
            return sharding.gather_heads_inplace(self.full)
        Bc = self.q.shape[0] // self.chunks
        works, views = [], []
        e0.record(st)
        for c in range(self.chunks):
            sl = slice(c * Bc, (c + 1) * Bc)
            G.fused_tree_verify(self.q[sl], self.k[sl], self.v[sl], self.par_t[sl], max_depth=self.max_depth,
                                out=self.locals[c])
            view, work = sharding.gather_heads_inplace(self.fulls[c], async_op=True)
            views.append(view)
            works.append(work)
        e1.record(st)  # all attention chunks queued (the gathers overlap them on NCCL's stream)
        self.kernel_events.append((e0, e1))
        for w in works:
            if w is not None:
                w.wait()
        return views

    def post(self, o):
        """The output gather of one e2e step (a fresh buffer per step)."""
        return sharding.gather_heads(o)

    @property
    def lockstep(self) -> bool:
        """With the fused gather each step waits for the other ranks' rows."""
        return self.gather == "fused" and self.world > 1

    @property
    def persistent_out(self) -> bool:
        """End-to-end steps write the peer buffers (``e2e_step``), not a fresh tensor."""
        return self.gather == "fused"

    def e2e_step(self, k: int, q_d: torch.Tensor, par_d: torch.Tensor):
        """(fused gather) One end-to-end step's attention into buffer set k:
        the returned ``[B, Hq, N, D]`` view is the layer on this rank."""
        peer = self.peers[k]
        G.fused_tree_verify(q_d, self.k, self.v, out=peer.local, peer_group=peer,
                            **dict(self.kwargs(), parents=par_d))
        return peer.full

    def close(self):
        for p in self.peers:
            p.close()
        self.peers = []

    mode = "heads"
    graphable = False  # with --gather nccl the step holds an all-gather: timed eagerly

    def extra(self, world: int, ms_step: float) -> dict:
        if self.gather == "fused":
            return {"us_per_layer": round(ms_step * 1e3, 2), "gather": "fused into the attention epilogue "
                    "(NVLink stores to every rank's buffer, on-device completion counters)",
                    "tokens_verified_per_s": round(self.tokens / (ms_step * 1e-3), 1)}
        ev = self.kernel_events
        torch.cuda.synchronize(self.dev)
        k_ms = float(np.mean([a.elapsed_time(b) for a, b in ev])) if ev else float("nan")
        return {"us_per_layer": round(ms_step * 1e3, 2), "gather": "NCCL all-gather", "kernel_only_us": round(k_ms * 1e3, 2),
                "allgather_us": round((ms_step - k_ms) * 1e3, 2),
                "tokens_verified_per_s": round(self.tokens / (ms_step * 1e-3), 1)}


def _fill_normal(t: torch.Tensor, gen: torch.Generator, std: float) -> None:
    """Fills a bf16/fp32 tensor with N(0, std) in 64 MB fp32 pieces."""
    flat = t.view(-1)
    step = 1 << 24
    for s0 in range(0, flat.numel(), step):
        n = min(step, flat.numel() - s0)
        flat[s0:s0 + n] = (torch.randn(n, device=t.device, generator=gen) * std).to(t.dtype)


class VerifyWorkload:
    """One decode step's tree verification (the fused verifier kernel):
    logits [B, N + 1, V] bf16 ~ N(0, 2) (row 0 for the root, row 1 + t for
    node t), random 64-node trees, drafts uniform over the vocabulary except
    that about a quarter of the nodes, taken along random root-to-leaf paths
    from the root, carry the argmax of their row, so accepted paths of every
    length occur."""

    metric = "tree verifier HBM GB/s (logits bytes / step time)"
    graphable = True  # one stream-ordered public call, no host sync
    data = "synthetic (seeded N(0,2) bf16 logits, random trees, drafts 1/4 on argmax paths)"
    bound = "hbm"

    def __init__(self, name: str, dev: torch.device, first_seq: int = 0):
        cfg = WORKLOADS[name]
        self.name, self.cfg, self.dev = name, cfg, dev
        B, N, V = cfg["B"], cfg["N"], cfg["V"]
        R = N + 1
        rngs = [random.Random(2_000_003 + first_seq + j) for j in range(B)]
        self.parents = [random_tree(N, r, cfg["max_depth"]) for r in rngs]
        self.logits = torch.empty(B, R, V, device=dev, dtype=torch.bfloat16)
        draft = torch.empty(B, N, dtype=torch.int64)
        for j in range(B):
            gen = torch.Generator(device=dev).manual_seed(3_000_003 + first_seq + j)
            _fill_normal(self.logits[j], gen, 2.0)
            pred = self.logits[j].float().argmax(-1).cpu()
            g_cpu = torch.Generator().manual_seed(3_000_003 + first_seq + j)
            draft[j] = torch.randint(0, V, (N,), generator=g_cpu)
            par = self.parents[j]
            children = [[] for _ in range(N)]
            for t, p in enumerate(par):
                if p >= 0:
                    children[p].append(t)
            marked, r = set(), rngs[j]
            for _ in range(64 * N):
                if len(marked) >= N // 4:
                    break
                t = 0
                while True:
                    marked.add(t)
                    if not children[t] or len(marked) >= N // 4:
                        break
                    t = r.choice(children[t])
            for t in marked:
                draft[j, t] = pred[0 if par[t] < 0 else 1 + par[t]]
        self.draft = draft.to(device=dev, dtype=torch.int32)
        self.par_t = torch.tensor(self.parents, dtype=torch.int32, device=dev)
        self.bytes = (B * R * V * 2 + 2 * B * N * 4                     # logits, draft, parents
                      + B * (R * 4 + N * 4 + 4 * 4))                    # pred, path, 4 per-sequence outputs
        self.flops = 0
        self.tokens = B * N

    def step(self):
        return G.verify_tree(self.logits, self.draft, self.par_t)

    def plan(self):
        return {"backend": "verify_kernel", "splits": None, "launches": 1}

    def config(self, world: int, plan: dict) -> dict:
        cfg = self.cfg
        return {"workload": self.name, "batch_per_gpu": cfg["B"], "tree_nodes": cfg["N"],
                "logits_rows": cfg["N"] + 1, "vocab": cfg["V"], "logits_dtype": "bf16",
                "parallelism": f"sequence-sharded x{world}" if world > 1 else "single GPU",
                "l2": f"inputs larger than L2 ({self.bytes / 1e6:.0f} MB per step per GPU)",
                "backend": plan["backend"]}

    def extra(self, world: int, ms_step: float) -> dict:
        return {"us_per_step": round(ms_step * 1e3, 2),
                "trees_verified_per_s": round(world * self.cfg["B"] / (ms_step * 1e-3), 1)}

    def e2e(self, steps: int, warmup: int, world: int):
        """Each step: drafts and parents in from pinned host memory, the
        verifier, accepted lengths, paths and bonus tokens back out (the
        logits stay on the device, where the model wrote them)."""
        dev = self.dev
        dr_h, par_h = self.draft.cpu().pin_memory(), self.par_t.cpu().pin_memory()
        dr_d, par_d = torch.empty_like(self.draft), torch.empty_like(self.par_t)
        B, N = self.cfg["B"], self.cfg["N"]
        len_h = torch.empty(B, dtype=torch.int32).pin_memory()
        path_h = torch.empty(B, N, dtype=torch.int32).pin_memory()
        bonus_h = torch.empty(B, dtype=torch.int32).pin_memory()
        h2d = (dr_h.numel() + par_h.numel()) * 4
        d2h = (len_h.numel() + path_h.numel() + bonus_h.numel()) * 4

        def one():
            dr_d.copy_(dr_h, non_blocking=True)
            par_d.copy_(par_h, non_blocking=True)
            r = G.verify_tree(self.logits, dr_d, par_d)
            len_h.copy_(r.accepted_len, non_blocking=True)
            path_h.copy_(r.path, non_blocking=True)
            bonus_h.copy_(r.bonus, non_blocking=True)

        ms = _time_loop(one, dev, steps, warmup, world)
        return ms, h2d, d2h, "logits resident in HBM (written there by the model); drafts and parents in, results out"

    def cpu_baseline(self, budget_s: float):
        from oracle import gorgon_oracle as O
        B = self.cfg["B"]
        times = []
        t_start = time.perf_counter()
        for j in range(B):
            lg = self.logits[j].float().cpu().numpy()
            dr = self.draft[j].cpu().tolist()
            t0 = time.perf_counter()
            O.verify_tree(lg, dr, self.parents[j])
            times.append(time.perf_counter() - t0)
            if time.perf_counter() - t_start > budget_s:
                break
        step_s = float(np.mean(times)) * B
        return {"value": round(self.bytes / step_s / 1e9, 4), "unit": "GB/s", "cores": 1, "kind": "port",
                "us_per_step": round(step_s * 1e6, 1),
                "sample": (f"{len(times)} of {B} sequences through the oracle's verify_tree (numpy argmax "
                           f"over all rows, then the path walk), extrapolated to the batch")}


class TrimWorkload:
    """Trim-on-reject after verification: for every layer, sequence and kv
    head, the accepted path's K/V rows (root included, <= 6) move to the slots
    right after the prefix, in place, in one launch over all layers."""

    metric = "KV trim HBM GB/s (rows moved, read + write, / step time)"
    graphable = True  # one stream-ordered public call (the layer pointers go by value)
    flush_l2 = True  # the ~22 MB of rows a step moves fit in L2
    data = "synthetic (seeded N(0,1) bf16 caches, random trees, random accepted paths)"
    bound = "hbm"

    def __init__(self, name: str, dev: torch.device, first_seq: int = 0):
        from projectgorgon_b200.inference.kv_cache import GorgonKVCache
        cfg = WORKLOADS[name]
        self.name, self.cfg, self.dev = name, cfg, dev
        B, Ly, H, D, P, N = cfg["B"], cfg["layers"], cfg["Hkv"], cfg["D"], cfg["P"], cfg["N"]
        S = P + N
        gen = torch.Generator(device=dev).manual_seed(4_000_003 + first_seq)
        layers = []
        for _ in range(Ly):
            k = torch.empty(B, H, S, D, device=dev, dtype=torch.bfloat16)
            v = torch.empty_like(k)
            _fill_normal(k, gen, 1.0)
            _fill_normal(v, gen, 1.0)
            layers.append((k, v))
        self.cache = GorgonKVCache()
        self.cache.update(tuple(layers))
        rngs = [random.Random(5_000_003 + first_seq + j) for j in range(B)]
        idx = torch.zeros(B, cfg["max_depth"] + 1, dtype=torch.int32)
        lens = torch.zeros(B, dtype=torch.int32)
        for j, r in enumerate(rngs):
            par = random_tree(N, r, cfg["max_depth"])
            children = [[] for _ in range(N)]
            for t, p in enumerate(par):
                if p >= 0:
                    children[p].append(t)
            path, t = [0], 0
            while children[t] and r.random() < 0.8:
                t = r.choice(children[t])
                path.append(t)
            lens[j] = len(path)
            idx[j, :len(path)] = torch.tensor([P + t for t in path], dtype=torch.int32)
        self.idx, self.lens = idx.to(dev), lens.to(dev)
        self.moved_rows = int(lens.sum())
        self.bytes = 2 * 2 * self.moved_rows * H * D * 2 * Ly   # read + write of K and V rows
        self.flops = 0
        self.tokens = self.moved_rows

    def step(self):
        self.cache.trim(self.idx, self.lens, dst_start=self.cfg["P"])

    def plan(self):
        return {"backend": "kv_trim_kernel", "splits": None, "launches": 1}

    def config(self, world: int, plan: dict) -> dict:
        cfg = self.cfg
        return {"workload": self.name, "batch_per_gpu": cfg["B"], "layers": cfg["layers"],
                "heads_kv": cfg["Hkv"], "head_dim": cfg["D"], "prefix": cfg["P"],
                "cache_seq": cfg["P"] + cfg["N"], "rows_moved_per_layer": self.moved_rows,
                "parallelism": f"sequence-sharded x{world}" if world > 1 else "single GPU",
                "l2": f"each step moves scattered rows of a {2 * cfg['layers'] * cfg['B'] * cfg['Hkv'] * (cfg['P'] + cfg['N']) * cfg['D'] * 2 / 1e9:.1f} GB cache",
                "backend": plan["backend"]}

    def extra(self, world: int, ms_step: float) -> dict:
        return {"us_per_step": round(ms_step * 1e3, 2)}

    def e2e(self, steps: int, warmup: int, world: int):
        """Each step: the accepted source rows and lengths in from pinned host
        memory, the trim, and the lengths back out."""
        dev = self.dev
        idx_h, lens_h = self.idx.cpu().pin_memory(), self.lens.cpu().pin_memory()
        idx_d, lens_d = torch.empty_like(self.idx), torch.empty_like(self.lens)
        out_h = torch.empty_like(lens_h).pin_memory()
        h2d = (idx_h.numel() + lens_h.numel()) * 4
        d2h = out_h.numel() * 4

        def one():
            idx_d.copy_(idx_h, non_blocking=True)
            lens_d.copy_(lens_h, non_blocking=True)
            self.cache.trim(idx_d, lens_d, dst_start=self.cfg["P"])
            out_h.copy_(lens_d, non_blocking=True)

        ms = _time_loop(one, dev, steps, warmup, world)
        return ms, h2d, d2h, "cache resident in HBM; accepted rows and lengths in, lengths out"

    def cpu_baseline(self, budget_s: float):
        """The reference algorithm (clone of each layer's cache, then the row
        gather: ``apply_cache_slice``) through the oracle on one layer of a few
        sequences, extrapolated to all layers and sequences."""
        from oracle import gorgon_oracle as O
        cfg = self.cfg
        nb = 4
        k = self.cache.past_key_values[0][0][:nb].float().cpu().numpy()
        v = self.cache.past_key_values[0][1][:nb].float().cpu().numpy()
        idx = self.idx[:nb].cpu().numpy()
        lens = self.lens[:nb].cpu().numpy()
        ds = np.full(nb, cfg["P"], dtype=np.int64)
        times = []
        t_start = time.perf_counter()
        while time.perf_counter() - t_start < min(budget_s, 5.0) or not times:
            t0 = time.perf_counter()
            O.kv_trim([(k, v)], idx, lens, ds)
            times.append(time.perf_counter() - t0)
        step_s = float(np.mean(times)) * (cfg["B"] / nb) * cfg["layers"]
        return {"value": round(self.bytes / step_s / 1e9, 4), "unit": "GB/s", "cores": 1, "kind": "port",
                "us_per_step": round(step_s * 1e6, 1),
                "sample": (f"one layer of {nb} sequences through the oracle's kv_trim (the reference's "
                           f"clone + gather), {len(times)} runs, extrapolated to {cfg['layers']} layers and "
                           f"{cfg['B']} sequences")}


class CandidateWorkload:
    """Candidate-tree construction for a batch (gorgon_candidate_tree): the
    Medusa heads' logits [B, heads, V] bf16 ~ N(0, 2) are read once for every
    head's top-k, softmax and entropy, then each sequence's tree is assembled
    under the node budget."""

    metric = "candidate-tree builder HBM GB/s (logits bytes / step time)"
    graphable = True  # stream-ordered public call: three launches, workspace from torch's allocator
    data = "synthetic (seeded N(0,2) bf16 head logits)"
    bound = "hbm"
    flush_l2 = True  # 33 MB of logits fit in L2

    def __init__(self, name: str, dev: torch.device, first_seq: int = 0):
        cfg = WORKLOADS[name]
        self.name, self.cfg, self.dev = name, cfg, dev
        B, L, V = cfg["B"], cfg["heads"], cfg["V"]
        self.logits = torch.empty(B, L, V, device=dev, dtype=torch.bfloat16)
        for j in range(B):
            _fill_normal(self.logits[j], torch.Generator(device=dev).manual_seed(4_000_003 + first_seq + j), 2.0)
        self.cap = G.inference.max_tree_nodes(cfg["top_k"], L, V, cfg["max_candidates"])
        self.bytes = B * L * V * 2 + B * (self.cap * (8 + 4 + 4) + 4)  # logits in; tokens, parents, probs, count out
        self.flops = 0
        self.tokens = B * self.cap

    def step(self):
        c = self.cfg
        return G.build_candidate_trees(self.logits, top_k=c["top_k"], max_candidates=c["max_candidates"])

    def plan(self):
        return {"backend": "cand_segment_kernel", "splits": None, "launches": 3}

    def config(self, world: int, plan: dict) -> dict:
        c = self.cfg
        return {"workload": self.name, "batch_per_gpu": c["B"], "heads": c["heads"], "vocab": c["V"],
                "top_k": c["top_k"], "max_candidates": c["max_candidates"], "logits_dtype": "bf16",
                "parallelism": f"sequence-sharded x{world}" if world > 1 else "single GPU",
                "l2": "L2 flushed before every step (a 256 MB write outside the step's events)",
                "backend": plan["backend"]}

    def extra(self, world: int, ms_step: float) -> dict:
        return {"us_per_step": round(ms_step * 1e3, 2),
                "trees_built_per_s": round(world * self.cfg["B"] / (ms_step * 1e-3), 1)}

    def e2e(self, steps: int, warmup: int, world: int):
        """Each step: the trees built and their tokens, parents and node
        counts copied to pinned host memory (the logits stay on the device,
        where the heads wrote them)."""
        dev, B = self.dev, self.cfg["B"]
        tok_h = torch.empty(B, self.cap, dtype=torch.int64).pin_memory()
        par_h = torch.empty(B, self.cap, dtype=torch.int32).pin_memory()
        n_h = torch.empty(B, dtype=torch.int32).pin_memory()
        d2h = tok_h.numel() * 8 + par_h.numel() * 4 + n_h.numel() * 4

        def one():
            t = self.step()
            tok_h.copy_(t.tokens, non_blocking=True)
            par_h.copy_(t.parents, non_blocking=True)
            n_h.copy_(t.n_nodes, non_blocking=True)

        ms = _time_loop(one, dev, steps, warmup, world)
        return ms, 0, d2h, "head logits resident in HBM (written there by the heads); trees out to the host"

    def cpu_baseline(self, budget_s: float):
        from oracle import gorgon_oracle as O
        c = self.cfg
        times = []
        t_start = time.perf_counter()
        for j in range(c["B"]):
            lg = self.logits[j].float().cpu().numpy()
            t0 = time.perf_counter()
            levels = [O.head_topk(lg[h], c["top_k"]) for h in range(c["heads"])]
            O.build_candidate_tree(levels, c["top_k"], max_candidates=c["max_candidates"])
            times.append(time.perf_counter() - t0)
            if time.perf_counter() - t_start > budget_s:
                break
        step_s = float(np.mean(times)) * c["B"]
        return {"value": round(self.bytes / step_s / 1e9, 4), "unit": "GB/s", "cores": 1, "kind": "port",
                "us_per_step": round(step_s * 1e6, 1),
                "sample": (f"{len(times)} of {c['B']} sequences through the oracle's head_topk (per head: "
                           f"top-k, softmax, entropy) and build_candidate_tree, extrapolated to the batch")}


class HeadsWorkload:
    """Candidate trees from the Medusa heads' last Linear with the logits
    never stored (gorgon_head_candidate_tree): every head's lm_head weight
    [V, H] bf16 streams from HBM once per step, the logits of the batch's
    head inputs are computed and reduced to top-k, softmax and entropy in the
    same kernel, then the trees are assembled.  The weights (4.2 GB) are far
    larger than L2, so no flush is needed between steps."""

    metric = "fused Medusa heads HBM GB/s (lm_head weight bytes / step time)"
    graphable = True  # stream-ordered public call (the weight pointers go by value)
    data = "synthetic (seeded N(0, 0.02) bf16 lm_head weights, N(0, 1) bf16 head inputs)"
    bound = "hbm"
    flush_l2 = False

    def __init__(self, name: str, dev: torch.device, first_seq: int = 0):
        cfg = WORKLOADS[name]
        self.name, self.cfg, self.dev = name, cfg, dev
        B, L, H, V = cfg["B"], cfg["heads"], cfg["H"], cfg["V"]
        self.w = []
        for l in range(L):
            w = torch.empty(V, H, device=dev, dtype=torch.bfloat16)
            _fill_normal(w, torch.Generator(device=dev).manual_seed(5_000_011 + l), 0.02)
            self.w.append(w)
        self.x = torch.empty(B, L, H, device=dev, dtype=torch.bfloat16)
        for j in range(B):
            _fill_normal(self.x[j], torch.Generator(device=dev).manual_seed(6_000_007 + first_seq + j), 1.0)
        self.cap = G.inference.max_tree_nodes(cfg["top_k"], L, V, cfg["max_candidates"])
        self.bytes = L * V * H * 2 + B * L * H * 2 + B * (self.cap * (8 + 4 + 4) + 4)
        self.flops = 2 * B * L * V * H
        self.tokens = B * self.cap

    def step(self):
        c = self.cfg
        return G.inference.head_candidate_trees(self.x, self.w, top_k=c["top_k"], max_candidates=c["max_candidates"])

    def plan(self):
        return {"backend": "head_segment_kernel", "splits": None, "launches": 3}

    def config(self, world: int, plan: dict) -> dict:
        c = self.cfg
        return {"workload": self.name, "batch_per_gpu": c["B"], "heads": c["heads"], "hidden": c["H"],
                "vocab": c["V"], "top_k": c["top_k"], "max_candidates": c["max_candidates"],
                "weights_dtype": "bf16", "logits_dtype": "bf16 (rounded in the kernel, never stored)",
                "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                "l2": "inputs larger than L2 (4.2 GB of weights per step)", "backend": plan["backend"]}

    def extra(self, world: int, ms_step: float) -> dict:
        c = self.cfg
        out = {"us_per_step": round(ms_step * 1e3, 2),
               "trees_built_per_s": round(world * c["B"] / (ms_step * 1e-3), 1)}
        # the same step unfused: cuBLAS GEMMs write the logits, the candidate kernels read them
        L = c["heads"]

        def unfused():
            lg = torch.stack([self.x[:, l] @ self.w[l].T for l in range(L)], dim=1)
            return G.build_candidate_trees(lg, top_k=c["top_k"], max_candidates=c["max_candidates"])
        ms_u = _time_loop(unfused, self.dev, 10, 3, 1) / 10
        out["unfused_us_per_step"] = round(ms_u * 1e3, 2)
        return out

    def e2e(self, steps: int, warmup: int, world: int):
        """Each step: the head inputs copied in from pinned host memory, the
        trees built, their tokens, parents and node counts copied out (the
        weights stay resident, as a model's do)."""
        B, L, H = self.cfg["B"], self.cfg["heads"], self.cfg["H"]
        x_h = self.x.cpu().pin_memory()
        tok_h = torch.empty(B, self.cap, dtype=torch.int64).pin_memory()
        par_h = torch.empty(B, self.cap, dtype=torch.int32).pin_memory()
        n_h = torch.empty(B, dtype=torch.int32).pin_memory()
        d2h = tok_h.numel() * 8 + par_h.numel() * 4 + n_h.numel() * 4

        def one():
            self.x.copy_(x_h, non_blocking=True)
            t = self.step()
            tok_h.copy_(t.tokens, non_blocking=True)
            par_h.copy_(t.parents, non_blocking=True)
            n_h.copy_(t.n_nodes, non_blocking=True)

        ms = _time_loop(one, self.dev, steps, warmup, world)
        return ms, B * L * H * 2, d2h, "lm_head weights resident in HBM; head inputs in, trees out through pinned host memory"

    def cpu_baseline(self, budget_s: float):
        return heads_cpu_sample(self.cfg, budget_s)


def heads_cpu_sample(cfg: dict, budget_s: float) -> dict:
    """The oracle on the host: head_logits (float64 matrix-vector products
    through numpy's BLAS) over a 16384-row slice of one head's weights,
    extrapolated to every row of every head and sequence, plus one
    sequence's head_topk and build_candidate_tree on full-width logits."""
    from oracle import gorgon_oracle as O
    B, L, H, V, k, mc = cfg["B"], cfg["heads"], cfg["H"], cfg["V"], cfg["top_k"], cfg["max_candidates"]
    rng = np.random.default_rng(0)
    rows = 16384
    w = rng.standard_normal((rows, H)) * 0.02
    x = rng.standard_normal((1, H))
    lg_full = rng.standard_normal((L, V), dtype=np.float32) * 2.0
    t_g, t_c, n = [], [], 0
    t_start = time.perf_counter()
    while n < 3 or time.perf_counter() - t_start < min(budget_s, 5.0):
        t0 = time.perf_counter()
        O.head_logits(x, [w], "bf16")
        t_g.append(time.perf_counter() - t0)
        t0 = time.perf_counter()
        levels = [O.head_topk(lg_full[h], k) for h in range(L)]
        O.build_candidate_tree(levels, k, max_candidates=mc)
        t_c.append(time.perf_counter() - t0)
        n += 1
        if time.perf_counter() - t_start > budget_s:
            break
    step_s = (float(np.mean(t_g)) * (V / rows) * L + float(np.mean(t_c))) * B
    wl_bytes = L * V * H * 2 + B * L * H * 2 + B * (min(sum(k ** (i + 1) for i in range(L)), mc) * 16 + 4)
    return {"value": round(wl_bytes / step_s / 1e9, 4), "unit": "GB/s", "cores": blas_threads(), "kind": "port",
            "us_per_step": round(step_s * 1e6, 1),
            "sample": (f"{n} runs of the oracle's head_logits over a {rows}-row slice of one head (float64 "
                       f"BLAS), extrapolated to {L} heads x {V} rows x {B} sequence(s), plus head_topk and "
                       f"build_candidate_tree of one sequence")}


def make_workload(name: str, dev: torch.device, first_seq: int = 0):
    kind = WORKLOADS[name].get("kind", "attn")
    return {"attn": Workload, "verify": VerifyWorkload, "trim": TrimWorkload,
            "cand": CandidateWorkload, "heads": HeadsWorkload}[kind](name, dev, first_seq)


# --------------------------------------------------------------------------
# clocks during the timed region
# --------------------------------------------------------------------------
class ClockSampler:
    """Samples SM clock and clock-event reasons of one GPU every 0.5 ms while
    the timed region runs (NVML), so that even a timed region of a few
    milliseconds carries several samples."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, dev: torch.device, period_s: float = 0.0005):
        self.dev, self.period = dev, period_s
        self.samples = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._nvml = None
        self._sample = None
        self._last_poll = 0.0

    def _handle(self):
        import pynvml
        pynvml.nvmlInit()
        self._nvml = pynvml
        try:
            pr = torch.cuda.get_device_properties(self.dev)
            bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
            return pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml.nvmlDeviceGetHandleByIndex(self.dev.index or 0)

    def __enter__(self):
        try:
            h = self._handle()
            nv = self._nvml
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons",
                                  getattr(nv, "nvmlDeviceGetCurrentClocksThrottleReasons", None))

            def sample():
                try:
                    mhz = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                    rs = int(get_reasons(h)) if get_reasons else 0
                    self.samples.append((mhz, rs))
                except Exception:
                    pass

            def run():
                while not self._stop.is_set():
                    sample()
                    self._stop.wait(self.period)

            # the first reads of a process take milliseconds (measured: up to
            # 5 ms, then about 1 us each): made here, outside the timed region
            for _ in range(3):
                sample()
            self.samples.clear()
            self._sample = sample
            self._thread = threading.Thread(target=run, daemon=True)
            self._thread.start()
        except Exception as exc:  # pragma: no cover - NVML missing
            log(f"clock sampling unavailable: {exc}")
        return self

    def poll(self, force: bool = False):
        """One sample from the calling thread, at most one per sampling period
        unless `force` (the timing loop samples after it has queued every
        step, while the GPU works through them)."""
        now = time.perf_counter()
        if self._sample is not None and (force or now - self._last_poll >= self.period):
            self._last_poll = now
            self._sample()

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        mhz = [m for m, _ in self.samples]
        reasons = set()
        for _, rs in self.samples:
            for bit, name in self.REASONS.items():
                if rs & bit:
                    reasons.add(name)
        return {"sm_mhz": float(np.median(mhz)), "sm_max_mhz": self.max_mhz, "reasons": sorted(reasons),
                "samples": len(self.samples), "source": "nvml"}


# --------------------------------------------------------------------------
# CPU baseline: the reference's attention on whole sequences, host cores
# --------------------------------------------------------------------------
def use_all_host_threads() -> None:
    """Lets numpy's BLAS use every host thread (torchrun sets OMP_NUM_THREADS=1
    for each rank; the reference arm runs on rank 0 alone)."""
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(os.cpu_count() or 1)
    except Exception:  # pragma: no cover
        pass


def blas_threads() -> int:
    try:
        from threadpoolctl import threadpool_info
        return max(int(i.get("num_threads", 1)) for i in threadpool_info()) or 1
    except Exception:  # pragma: no cover
        return os.cpu_count() or 1


def cpu_baseline(wl: "Workload", budget_s: float = 12.0):
    """The reference's mask + attention (``HostAttention``) on whole sequences
    of the workload, run one after another on the host cores until about
    `budget_s` seconds have passed (at least one sequence); the rate is the
    bytes of the sequences run over the time they took."""
    ha = HostAttention(wl.name)
    ha.run_seq(0)  # warm-up
    done, secs, nbytes = 0, 0.0, 0
    while done < wl.cfg["B"] and (done == 0 or secs < budget_s):
        ha.seq_inputs(done)  # drawn outside the timed call
        t0 = time.perf_counter()
        ha.run_seq(done)
        secs += time.perf_counter() - t0
        nbytes += ha.seq_bytes(done)
        done += 1
    return {
        "value": round(nbytes / secs / 1e9, 4),
        "unit": "GB/s",
        "cores": ha.cores,
        "kind": ha.kind,
        "us_per_layer": round(secs / done * wl.cfg["B"] * 1e6, 1),
        "sample": (f"{done} of the {wl.cfg['B']} sequences of this workload (all {wl.cfg['Hq']} query heads), "
                   f"{ha.origin} with its build_tree_mask on {ha.cores} host threads; us_per_layer scales "
                   f"the measured time to the whole batch"),
    }


# --------------------------------------------------------------------------
# timing
# --------------------------------------------------------------------------
def dist_setup():
    env = sharding.dist_env()
    return env.world, env.rank, env.local_rank


def capture_step(wl, dev):
    """A CUDA graph of one step (the public call, captured once on a side
    stream as torch requires), replayed for each timed step: the way a
    serving loop runs a launch-bound step, without the per-call host path
    and driver launch cost in the device time."""
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for _ in range(2):
            wl.step()
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        wl.step()
    return g


def time_device(wl: Workload, steps: int, warmup: int, world: int, graph: bool = False):
    """(ms of the timed steps, mean ms per step, clock summary).  A workload
    whose inputs fit in L2 sets ``flush_l2``: a 256 MB write then evicts L2
    before every step, outside the step's events, and the time is the sum of
    the steps' own event times.  With `graph`, each step replays a CUDA graph
    of the step (see capture_step); the warm-up steps run eagerly first."""
    dev = wl.dev
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev) if getattr(wl, "flush_l2", False) else None
    for _ in range(warmup):
        wl.step()
    torch.cuda.synchronize(dev)
    if hasattr(wl, "kernel_events"):
        wl.kernel_events.clear()  # only the timed steps' attention events count
    step = wl.step
    g = None
    if graph:
        try:
            g = capture_step(wl, dev)
        except RuntimeError as exc:  # a capture the runtime refuses: time eager calls instead
            log(f"CUDA-graph capture failed ({exc}); timing eager calls")
            wl.graph_failed = True
        if g is not None:
            step = g.replay
            for _ in range(2):
                step()
        torch.cuda.synchronize(dev)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(dev)
    st = torch.cuda.current_stream(dev)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    with ClockSampler(dev) as clk:
        if getattr(wl, "lockstep", False):
            # ranks whose steps wait on one another on the device: one more
            # untimed step queued right before the timed ones, so that every
            # rank's timed region starts when that step's handshake releases
            # it, not when its host left the barrier
            step()
        for i in range(steps):
            if flush is not None:
                flush.fill_(i & 0xff)
            starts[i].record(st)
            step()
            ends[i].record(st)
        # every step is queued: sample the clocks while the GPU works through
        # them (a read takes about a microsecond, but an occasional one takes
        # milliseconds, which between launches would leave the GPU waiting)
        clk.poll(force=True)
        while not ends[-1].query():
            clk.poll(force=True)
        torch.cuda.synchronize(dev)
    total_ms = starts[0].elapsed_time(ends[-1])
    per = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    if flush is not None:
        total_ms = float(np.sum(per))
    del g
    if world > 1:
        torch.distributed.barrier()
    return total_ms, float(np.mean(per)), clk.summary()


def time_e2e(wl: Workload, steps: int, warmup: int, world: int):
    """Each step: H2D of Q, the tree's K/V rows and parents from pinned host
    memory, the tree rows written into the resident cache, the attention
    call, and D2H of the output.  Steps are pipelined the way a serving loop
    overlaps transfers with compute: step i + 1's inputs are copied in on one
    stream while step i computes on another, and step i's output is copied out
    on a third; two sets of device input buffers alternate, and the copy-in is
    split over two streams.  The timed region
    starts before the first step's copy-in and ends after the last step's
    copy-out, so every step's transfers lie inside it."""
    dev = wl.dev
    cfg = wl.cfg
    B, N = cfg["B"], cfg["N"]
    q_h = wl.q.cpu().pin_memory()
    par_h = wl.par_t.cpu().pin_memory()
    if wl.ragged:
        rows = torch.cat([torch.arange(int(wl.cu[b + 1]) - N, int(wl.cu[b + 1])) for b in range(B)]).to(dev)
        kt_h = wl.k[rows].cpu().pin_memory()
        vt_h = wl.v[rows].cpu().pin_memory()
    else:
        P = wl.prefixes[0]
        kt_h = wl.k[:, :, P:P + N].contiguous().cpu().pin_memory()
        vt_h = wl.v[:, :, P:P + N].contiguous().cpu().pin_memory()
    nbuf = 2
    bufs = [(torch.empty_like(wl.q), torch.empty(kt_h.shape, dtype=kt_h.dtype, device=dev),
             torch.empty(vt_h.shape, dtype=vt_h.dtype, device=dev), torch.empty_like(wl.par_t))
            for _ in range(nbuf)]
    post = getattr(wl, "post", None)
    out_shape = wl.out.shape if post is not None else wl.q.shape
    outs_h = [torch.empty(out_shape, dtype=wl.q.dtype).pin_memory() for _ in range(nbuf)]
    h2d = sum(t.numel() * t.element_size() for t in (q_h, kt_h, vt_h, par_h))
    d2h = outs_h[0].numel() * outs_h[0].element_size()
    s_c = torch.cuda.current_stream(dev)
    # copy-in over two streams (Q on one, the tree's K/V rows and parents on the
    # other): a single stream's copies run on one copy engine, and one engine
    # does not fill the link (measured: 1,463 -> 1,626 GB/s end to end)
    s_in, s_in2, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    in_ready = [torch.cuda.Event() for _ in range(nbuf)]
    in_ready2 = [torch.cuda.Event() for _ in range(nbuf)]
    in_free = [torch.cuda.Event() for _ in range(nbuf)]
    done = [torch.cuda.Event() for _ in range(nbuf)]
    out_free = [torch.cuda.Event() for _ in range(nbuf)]
    kw = wl.kwargs()
    # per-step stamps of each stage, on the stream that runs it: copy-in (both
    # copy streams), compute (the tree rows' cache write and the attention),
    # copy-out; read after the loop, so they cost no synchronisation
    stamps = []

    def ev():
        return torch.cuda.Event(enable_timing=True)

    def one(i, rec):
        k = i % nbuf
        q_d, kt_d, vt_d, par_d = bufs[k]
        st = [ev() for _ in range(8)] if rec else None
        with torch.cuda.stream(s_in):
            if i >= nbuf:
                s_in.wait_event(in_free[k])  # step i - 2 has read this buffer set
            if rec:
                st[0].record(s_in)
            q_d.copy_(q_h, non_blocking=True)
            if rec:
                st[1].record(s_in)
            in_ready[k].record(s_in)
        with torch.cuda.stream(s_in2):
            if i >= nbuf:
                s_in2.wait_event(in_free[k])
            if rec:
                st[2].record(s_in2)
            kt_d.copy_(kt_h, non_blocking=True)
            vt_d.copy_(vt_h, non_blocking=True)
            par_d.copy_(par_h, non_blocking=True)
            if rec:
                st[3].record(s_in2)
            in_ready2[k].record(s_in2)
        s_c.wait_event(in_ready[k])
        s_c.wait_event(in_ready2[k])
        if rec:
            st[4].record(s_c)
        if wl.ragged:
            wl.k[rows] = kt_d
            wl.v[rows] = vt_d
        else:
            wl.k[:, :, P:P + N].copy_(kt_d)
            wl.v[:, :, P:P + N].copy_(vt_d)
        e2e_step = wl.e2e_step if getattr(wl, "persistent_out", False) else None
        if e2e_step is not None:
            # output in a persistent buffer (one per buffer set): written
            # again two steps later, once this step's copy-out has read it
            if i >= nbuf:
                s_c.wait_event(out_free[k])
            o = e2e_step(k, q_d, par_d)
        else:
            o = G.fused_tree_verify(q_d, wl.k, wl.v, **dict(kw, parents=par_d))
            if post is not None:
                o = post(o)
        if rec:
            st[5].record(s_c)
        in_free[k].record(s_c)
        done[k].record(s_c)
        with torch.cuda.stream(s_out):
            s_out.wait_event(done[k])
            if rec:
                st[6].record(s_out)
            outs_h[k].copy_(o, non_blocking=True)
            if rec:
                st[7].record(s_out)
            out_free[k].record(s_out)
            if e2e_step is None:
                o.record_stream(s_out)
        if rec:
            stamps.append(st)

    def run(n, rec):
        for i in range(n):
            one(i, rec)
        s_c.wait_stream(s_in)
        s_c.wait_stream(s_in2)
        s_c.wait_stream(s_out)

    run(warmup, False)
    torch.cuda.synchronize(dev)
    if world > 1:
        torch.distributed.barrier()
    if getattr(wl, "lockstep", False):
        wl.step()  # untimed: the ranks leave this step's handshake together (see time_device)
    e0, e1 = ev(), ev()
    e0.record(s_c)
    s_in.wait_event(e0)
    s_in2.wait_event(e0)
    s_out.wait_event(e0)
    t_host = time.perf_counter()
    run(steps, False)
    t_host = time.perf_counter() - t_host
    e1.record(s_c)
    torch.cuda.synchronize(dev)
    total = e0.elapsed_time(e1)
    # a second, instrumented pass gives each stage's own duration
    run(min(steps, 50), True)
    torch.cuda.synchronize(dev)
    cin = float(np.mean([max(a[0].elapsed_time(a[1]), a[2].elapsed_time(a[3])) for a in stamps]))
    comp = float(np.mean([a[4].elapsed_time(a[5]) for a in stamps]))
    cout = float(np.mean([a[6].elapsed_time(a[7]) for a in stamps]))
    parts = {"copy_in_ms": round(cin, 5), "compute_ms": round(comp, 5), "copy_out_ms": round(cout, 5),
             "host_issue_ms": round(t_host * 1e3 / steps, 5),
             "h2d_gbs": round(h2d / (cin * 1e-3) / 1e9, 2), "d2h_gbs": round(d2h / (cout * 1e-3) / 1e9, 2),
             "bound": max((("copy-in", cin), ("compute", comp), ("copy-out", cout),
                           ("host issue", t_host * 1e3 / steps)), key=lambda x: x[1])[0]}
    return total, h2d, d2h, parts


def _time_loop(one, dev, steps: int, warmup: int, world: int) -> float:
    """Device time (ms) of `steps` calls of `one` after `warmup` untimed ones."""
    for _ in range(warmup):
        one()
    torch.cuda.synchronize(dev)
    if world > 1:
        torch.distributed.barrier()
    st = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(steps):
        one()
    e1.record(st)
    torch.cuda.synchronize(dev)
    return e0.elapsed_time(e1)


def max_over_ranks(x: float, world: int, dev) -> float:
    return sharding.max_over_ranks(x, dev) if world > 1 else x


def peaks():
    """(HBM GB/s, burst bf16 TFLOP/s, source): measured on this pool's B200s
    when MEASURED_PEAKS.json is present, else the earlier pool measurement."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def run_ours(args):
    world, rank, local = dist_setup()
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    sharding.init(sharding.dist_env(), "nccl", dev, timeout_s=120)
    G.load_library()
    kind = WORKLOADS[args.workload].get("kind", "attn")
    if args.shard == "heads":
        if kind != "attn":
            raise SystemExit("--shard heads applies to the attention workloads")
        wl = HeadShardWorkload(args.workload, dev, rank, world, chunks=args.head_chunks, gather=args.gather)
    elif kind == "attn":
        # strong (default): the fixed batch split over the ranks; weak: a batch per rank
        mode = "weak" if args.shard == "weak" else "strong"
        first, count = seq_shard(args.workload, world, rank, mode)
        wl = Workload(args.workload, dev, first_seq=first, batch=count)
        wl.mode = mode
    else:
        # the other workloads run a whole batch per rank
        wl = make_workload(args.workload, dev, first_seq=rank * WORKLOADS[args.workload]["B"])
        wl.mode = "weak"
    plan = wl.plan()
    # bytes of the whole job: every rank's share (weak: every rank's batch)
    job_bytes = int(sharding.sum_over_ranks(wl.bytes, dev)) if world > 1 else wl.bytes
    graph = not args.eager and getattr(wl, "graphable", False)
    total_ms, launch_ms, clocks = time_device(wl, args.steps, args.warmup, world, graph=graph)
    total_ms = max_over_ranks(total_ms, world, dev)
    launch_ms = max_over_ranks(launch_ms, world, dev)
    e2e_steps = args.e2e_steps or max(100, args.steps)
    e2e = wl.e2e(e2e_steps, args.warmup, world)
    e2e_ms, h2d, d2h, e2e_note = e2e[:4]
    e2e_parts = e2e[4] if len(e2e) > 4 else None
    e2e_ms = max_over_ranks(e2e_ms, world, dev)
    extra = wl.extra(world, total_ms / args.steps)
    if hasattr(wl, "close"):
        wl.close()  # peer buffers: every rank unmaps and frees them together
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank != 0:
        return
    ms_step = total_ms / args.steps
    value = job_bytes * args.steps / (total_ms * 1e-3) / 1e9
    e2e_val = job_bytes * e2e_steps / (e2e_ms * 1e-3) / 1e9
    hbm_peak, tc_peak, peak_kind = peaks()
    if wl.bound == "tensor":
        achieved = wl.flops / (launch_ms * 1e-3) / 1e12
        roof = {"bound": "tensor", "achieved": round(achieved, 2), "peak": tc_peak, "unit": "TFLOP/s",
                "frac": round(achieved / tc_peak, 4),
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json bf16_tflops, burst)" if peak_kind == "measured"
                else "fallback 1590 TFLOP/s", "algorithmic_flops": wl.flops,
                "hbm_gbs": round(wl.bytes / (launch_ms * 1e-3) / 1e9, 2)}
    else:
        achieved = wl.bytes / (launch_ms * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": round(achieved, 2), "peak": hbm_peak, "unit": "GB/s",
                "frac": round(achieved / hbm_peak, 4),
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                else "fallback 6650 GB/s"}
        if wl.flops:
            roof["tflops"] = round(wl.flops / (launch_ms * 1e-3) / 1e12, 2)
    roof.update({"traffic": NCU_TRAFFIC_BYTES.get((wl.name, plan["backend"])) if world == 1 else None,
                 "launch_us": round(launch_ms * 1e3, 3), "algorithmic_bytes": wl.bytes,
                 "per": "one GPU's launch (the slowest rank's mean)" if world > 1 else "the launch"})
    e2e_out = {"value": round(e2e_val, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms / e2e_steps, 5), "steps": e2e_steps,
               "note": e2e_note}
    if e2e_parts:
        e2e_out.update(e2e_parts)
    out = {
        "metric": wl.metric,
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 5),
        "higher_is_better": True,
        "scaling": "weak" if wl.mode == "weak" else "strong",
        "vs_baseline": None,
        "dtype": wl.cfg["dtype"],
        "data": wl.data,
        "config": wl.config(world, plan),
        "plan": {"backend": plan["backend"], "splits": plan.get("splits"), "launches_per_step": plan["launches"],
                 "timed_as": ("CUDA graph of one step, replayed per step"
                              if graph and not getattr(wl, "graph_failed", False) else "eager public call per step")},
        "pct_of_8tbs": round(100.0 * value / world / 8000.0, 2),
        "roofline": roof,
        "e2e": e2e_out,
        "gpu_launches": plan["launches"] * args.steps,
        "clocks": clocks,
    }
    out.update(extra)
    if world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = wl.cpu_baseline(args.cpu_budget)
    print(json.dumps(out), flush=True)


def reference_attention():
    """(attention(q, k, v, mask), mask(parents, depth), kind, origin): the
    reference's own ``tree_attention_ref`` (torch on the host cores,
    ``src/gorgon/kernels/tree_attention_ref.py:8-18``) and ``build_tree_mask``
    (``src/gorgon/kernels/tree_mask.py:16-44``) from its unmodified install
    under ``baseline/_ref``; without that install, the oracle's numpy
    restatement of the same two functions."""
    ref_dir = ROOT / "baseline" / "_ref"
    if (ref_dir / "gorgon" / "kernels" / "tree_attention_ref.py").exists():
        if str(ref_dir) not in sys.path:
            sys.path.insert(0, str(ref_dir))
        from gorgon.kernels.tree_attention_ref import tree_attention_ref
        from gorgon.kernels.tree_mask import build_tree_mask

        def mask(parents, depth):
            return build_tree_mask(list(parents), depth=depth)
        return tree_attention_ref, mask, "reference", "the reference's tree_attention_ref (torch, fp32)"
    from oracle import gorgon_oracle as O

    def attn_np(q, k, v, m):
        return O.tree_attention(q.numpy(), k.numpy(), v.numpy(), m.numpy())

    def mask_np(parents, depth):
        return torch.from_numpy(O.build_tree_mask(parents, depth))
    return attn_np, mask_np, "port", "the oracle's tree_attention (numpy, fp32; reference install absent)"


def host_threads() -> int:
    """Every host thread for torch and BLAS (torchrun sets OMP_NUM_THREADS=1
    per rank; the reference arm runs on rank 0 alone)."""
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    use_all_host_threads()
    return n


class HostAttention:
    """The reference's verify attention on the host over whole sequences of
    an attention workload: per sequence its tree mask (``build_tree_mask``
    of the parents, ``max_depth`` hops, after a fully visible prefix), then
    ``tree_attention_ref`` for each query head over its kv head's P + N rows,
    in fp32 on the same seeded sequences the GPU arm runs (inputs drawn
    N(0, 1)/sqrt(d) and rounded to bf16 first for bf16 workloads)."""

    def __init__(self, name: str):
        self.name, self.cfg = name, WORKLOADS[name]
        self.attn, self.mask, self.kind, self.origin = reference_attention()
        self.cores = host_threads()
        self._cache = {}

    def seq_inputs(self, j: int):
        if j not in self._cache:
            cfg = self.cfg
            (P,), (par,) = attn_sequences(cfg, j, 1)
            N, D, Hq, Hkv = cfg["N"], cfg["D"], cfg["Hq"], cfg["Hkv"]
            g = torch.Generator().manual_seed(7_000_003 + j)
            s = 1.0 / math.sqrt(D)

            def draw(*shape):
                x = torch.randn(*shape, generator=g) * s
                return x.bfloat16().float() if cfg["dtype"] == "bf16" else x
            self._cache[j] = (draw(Hq, N, D), draw(Hkv, P + N, D), draw(Hkv, P + N, D), par, P)
        return self._cache[j]

    def run_seq(self, j: int) -> None:
        cfg = self.cfg
        q, k, v, par, P = self.seq_inputs(j)
        N, G_ = cfg["N"], cfg["Hq"] // cfg["Hkv"]
        tm = torch.as_tensor(self.mask(par, cfg["max_depth"]), dtype=torch.bool)
        m = torch.cat([torch.ones(N, P, dtype=torch.bool), tm], dim=1)
        for h in range(cfg["Hq"]):
            self.attn(q[h], k[h // G_], v[h // G_], m)

    def seq_bytes(self, j: int) -> int:
        return attn_bytes(self.cfg, [self.seq_inputs(j)[4]])

    def plan_step(self, target_s: float) -> int:
        """Sequences per step: as many whole sequences as fit in about
        `target_s` seconds (at least one, at most the batch)."""
        self.run_seq(0)
        t0 = time.perf_counter()
        self.run_seq(0)
        t_seq = time.perf_counter() - t0
        return int(max(1, min(self.cfg["B"], target_s // max(t_seq, 1e-6))))


def run_reference(args):
    """The reference arm on the host cores, same metric, workload and config
    as this build's arm.  Each step runs whole sequences of the workload --
    the full batch when it fits in about two seconds, else the first few --
    through the reference's own mask and attention functions, and is timed
    as it runs: nothing is extrapolated."""
    world, rank, _ = dist_setup()
    if rank != 0:
        return
    cfg = WORKLOADS[args.workload]
    if cfg.get("kind", "attn") != "attn":
        use_all_host_threads()
        run_reference_other(args, cfg, world)
        return
    ha = HostAttention(args.workload)
    per_step = ha.plan_step(2.0)
    seqs = list(range(per_step))
    for j in seqs:
        ha.seq_inputs(j)
    step_bytes = sum(ha.seq_bytes(j) for j in seqs)
    for _ in range(args.warmup):
        for j in seqs:
            ha.run_seq(j)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        for j in seqs:
            ha.run_seq(j)
        times.append(time.perf_counter() - t0)
    step_s = float(np.mean(times))
    value = step_bytes / step_s / 1e9
    mode = "weak" if args.shard == "weak" else ("heads" if args.shard == "heads" else "strong")
    what = (f"each step {per_step} of the {cfg['B']} sequences of the workload (all {cfg['Hq']} query heads "
            f"over each one's full prefix + tree): {ha.origin} with its build_tree_mask, on "
            f"{ha.cores} host threads, timed per step")
    out = {
        "impl": "reference",
        "metric": Workload.metric,
        "value": round(value, 4), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(step_s * 1e3, 3), "higher_is_better": True,
        "scaling": "weak" if mode == "weak" else "strong", "vs_baseline": None, "dtype": cfg["dtype"],
        "data": Workload.data,
        "config": attn_config(args.workload, world, mode, args.gather),
        "sequences_per_step": per_step,
        "us_per_layer": round(step_s * 1e6 * cfg["B"] / per_step, 1),
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": ha.cores, "kind": ha.kind,
                         "sample": what},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)


def run_reference_other(args, cfg: dict, world: int):
    """Reference arm of the verifier, trim and candidate-tree workloads: the
    oracle's verify_tree (one sequence per step), kv_trim (one layer of four
    sequences per step, the reference's clone + gather) or head_topk +
    build_candidate_tree (one sequence per step) on host-generated inputs of
    the workload's shapes, extrapolated to the whole step."""
    from oracle import gorgon_oracle as O
    rng = np.random.default_rng(0)
    prng = random.Random(0)
    B, N = cfg["B"], cfg.get("N", 0)
    if cfg["kind"] == "heads":
        for _ in range(max(args.warmup, 1)):
            heads_cpu_sample(cfg, 1.0)
        runs = [heads_cpu_sample(cfg, 5.0) for _ in range(args.steps)]
        step_us = float(np.mean([r["us_per_step"] for r in runs]))
        value = float(np.mean([r["value"] for r in runs]))
        cb = dict(runs[-1], value=round(value, 4))
        cb.pop("us_per_step", None)
        out = {
            "impl": "reference", "metric": HeadsWorkload.metric, "value": round(value, 4), "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_us / 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": cfg["dtype"],
            "data": "synthetic", "config": {"workload": args.workload, "batch_per_gpu": B},
            "cpu_baseline": cb,
            "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
        print(json.dumps(out), flush=True)
        return
    if cfg["kind"] == "cand":
        L, V, k, mc = cfg["heads"], cfg["V"], cfg["top_k"], cfg["max_candidates"]
        cap = min(sum(k ** (i + 1) for i in range(L)), mc)
        wl_bytes = B * L * V * 2 + B * (cap * 16 + 4)
        metric, what = CandidateWorkload.metric, ("one sequence through the oracle's head_topk and "
                                                  "build_candidate_tree, x batch")

        def sample():
            return rng.standard_normal((L, V), dtype=np.float32) * 2.0

        def run(s):
            levels = [O.head_topk(s[h], k) for h in range(L)]
            O.build_candidate_tree(levels, k, max_candidates=mc)
        scale = B
    elif cfg["kind"] == "verify":
        V, R = cfg["V"], cfg["N"] + 1
        wl_bytes = B * R * V * 2 + 2 * B * N * 4 + B * (R * 4 + N * 4 + 16)
        metric, what = VerifyWorkload.metric, "one sequence through the oracle's verify_tree, x batch"

        def sample():
            lg = rng.standard_normal((R, V), dtype=np.float32) * 2.0
            return lg, rng.integers(0, V, N).tolist(), random_tree(N, prng, cfg["max_depth"])

        def run(s):
            O.verify_tree(*s)
        scale = B
    else:
        nb, H, D, P = 4, cfg["Hkv"], cfg["D"], cfg["P"]
        S = P + N
        rows = 6 * B
        wl_bytes = 2 * 2 * rows * H * D * 2 * cfg["layers"]
        metric, what = TrimWorkload.metric, (f"one layer of {nb} sequences through the oracle's kv_trim "
                                             f"(clone + gather), x {B // nb} x {cfg['layers']} layers")

        def sample():
            k = rng.standard_normal((nb, H, S, D), dtype=np.float32)
            v = rng.standard_normal((nb, H, S, D), dtype=np.float32)
            idx = np.tile(np.arange(P, P + 6, dtype=np.int64), (nb, 1))
            return k, v, idx, np.full(nb, 6), np.full(nb, P)

        def run(s):
            k, v, idx, lens, ds = s
            O.kv_trim([(k, v)], idx, lens, ds)
        scale = (B / nb) * cfg["layers"]
    s = sample()
    for _ in range(args.warmup):
        run(s)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        run(s)
        times.append((time.perf_counter() - t0) * scale)
    step_s = float(np.mean(times))
    value = wl_bytes / step_s / 1e9
    out = {
        "impl": "reference", "metric": metric, "value": round(value, 4), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_s * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": cfg["dtype"],
        "data": "synthetic", "config": {"workload": args.workload, "batch_per_gpu": B},
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": 1, "kind": "port", "sample": what},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--e2e-steps", type=int, default=0,
                    help="steps of the e2e loop (default: the larger of --steps and 100)")
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD, choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--shard", default="sequences", choices=["sequences", "weak", "heads"],
                    help="multi-GPU split: the workload's batch divided by sequence over the ranks (strong "
                         "scaling, default), a whole batch per rank (weak scaling), or one layer's kv heads "
                         "per rank with the output gathered over NVLink (strong scaling)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--gather", choices=["fused", "nccl"], default="fused",
                    help="--shard heads: output gather fused into the attention (NVLink stores) or an NCCL all-gather")
    ap.add_argument("--head-chunks", type=int, default=1,
                    help="--shard heads: batch chunks whose all-gathers overlap the next chunk's attention")
    ap.add_argument("--eager", action="store_true",
                    help="time eager public calls per step instead of replaying a CUDA graph of the step")
    ap.add_argument("--cpu-budget", type=float, default=12.0)
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if ws != args.gpus:
        log(f"note: --gpus {args.gpus} but WORLD_SIZE={ws}; using WORLD_SIZE")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
