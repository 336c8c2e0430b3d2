"""Tree-verification benchmark: tree attention over [prefix | tree] on B200.

One step is one tree-verify attention layer over a batch of sequences, run
through the public operator ``fused_tree_verify`` (mask-free, parents only).
The default workload is the Llama-3-8B layer shape: batch 16, 32 query / 8
key-value heads, head_dim 128, prefix 8192, a 64-node random tree per
sequence (depth <= 5), bf16.

Prints one JSON line (rank 0).  ``value`` is algorithmic HBM GB/s summed over
all GPUs (K and V of every sequence read once, Q read once, output written
once, parents read once) with inputs resident in HBM; ``e2e`` is the same
metric with each step's new inputs (Q, the tree's K/V rows, parents) copied
from pinned host memory and the output copied back inside the timed region.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
    python bench.py --impl reference ...   # the CPU oracle port on host cores

Multi-GPU (torchrun, one rank per GPU): each rank verifies its own batch of
sequences (weak scaling by sequence); the timing is the max over ranks.
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
    # profiles/attn_tc_kernel_verify-b16-p8192-n64.md: 549.552 MB read + 3.763 MB written
    ("verify-b16-p8192-n64", "tcgen05"): 553314560,
    # profiles/attn_tc_kernel_verify-b1-p2048-n64.md: 9.273 MB read, 0 written
    ("verify-b1-p2048-n64", "tcgen05"): 9273088,
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


# --------------------------------------------------------------------------
# workload construction
# --------------------------------------------------------------------------
class Workload:
    """Seeded synthetic inputs of one workload, resident on `dev`.

    Sequence j of this rank is global sequence first_seq + j, and everything
    about it (prefix length, tree, q/k/v) comes from generators seeded by that
    global index, so the union of all ranks' shards is one well-defined job
    whatever the number of ranks."""

    def __init__(self, name: str, dev: torch.device, first_seq: int = 0):
        cfg = WORKLOADS[name]
        self.name, self.cfg, self.dev = name, cfg, dev
        B, Hq, Hkv, D, N = cfg["B"], cfg["Hq"], cfg["Hkv"], cfg["D"], cfg["N"]
        self.ragged = isinstance(cfg["P"], tuple)
        rngs = [random.Random(1_000_003 + first_seq + j) for j in range(B)]
        self.prefixes = [r.randint(*cfg["P"]) if self.ragged else cfg["P"] for r in rngs]
        self.parents = [make_tree(cfg, r) for r in rngs]
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
        esz = torch.tensor([], dtype=dt).element_size()
        kv_rows = sum(p + N for p in self.prefixes)
        self.bytes = (2 * kv_rows * Hkv * D * esz + 2 * B * Hq * N * D * esz + B * N * 4
                      + ((B + 1) * 4 if self.ragged else 0))
        self.flops = 4 * Hq * N * D * kv_rows
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

    def config(self, world: int, plan: dict) -> dict:
        cfg = self.cfg
        return {
            "workload": self.name, "batch_per_gpu": cfg["B"], "heads_q": cfg["Hq"], "heads_kv": cfg["Hkv"],
            "head_dim": cfg["D"], "prefix": cfg["P"] if not self.ragged else list(cfg["P"]),
            "tree_nodes": cfg["N"], "tree": cfg["tree"], "max_depth": self.max_depth,
            "mask": "parents (mask-free)",
            "parallelism": f"sequence-sharded x{world}" if world > 1 else "single GPU",
            "l2": ("L2 flushed before every step (a 256 MB write outside the step's events)" if self.flush_l2
                   else f"inputs larger than L2 ({self.bytes / 1e6:.0f} MB per step per GPU)"),
            "backend": plan["backend"], "splits": plan["splits"],
        }

    def extra(self, world: int, ms_step: float) -> dict:
        return {"us_per_layer": round(ms_step * 1e3, 2),
                "tokens_verified_per_s": round(world * self.tokens / (ms_step * 1e-3), 1)}

    def e2e(self, steps: int, warmup: int, world: int):
        ms, h2d, d2h = time_e2e(self, steps, warmup, world)
        return ms, h2d, d2h, ("prefix K/V cache resident in HBM; per step the tree's Q, K/V rows and "
                              "parents are copied in and the output copied out, pipelined: step i + 1's "
                              "copy-in and step i - 1's copy-out overlap step i's compute")

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

    def __init__(self, name: str, dev: torch.device, rank: int, world: int):
        cfg = WORKLOADS[name]
        if isinstance(cfg["P"], tuple):
            raise SystemExit("--shard heads needs a workload with one prefix length")
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
        self.out = torch.empty(B, Hq, N, D, device=dev, dtype=dt)
        esz = torch.tensor([], dtype=dt).element_size()
        # this rank's share: its K/V, Q and output slice, and the parents
        self.bytes = 2 * B * (h1 - h0) * L * D * esz + 2 * B * (q1 - q0) * N * D * esz + B * N * 4
        self.flops = 4 * (q1 - q0) * N * D * B * L
        self.tokens = B * N
        self.kernel_events = []

    def step(self):
        st = torch.cuda.current_stream(self.dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        o = G.fused_tree_verify(self.q, self.k, self.v, **self.kwargs())
        e1.record(st)
        self.kernel_events.append((e0, e1))
        return sharding.gather_heads(o, self.out)

    def post(self, o):
        """The output gather of one e2e step (a fresh buffer per step)."""
        return sharding.gather_heads(o)

    def config(self, world: int, plan: dict) -> dict:
        c = super().config(world, plan)
        c["parallelism"] = f"kv-head-sharded x{world}, NCCL all-gather of the output" if world > 1 else "single GPU"
        c["batch"] = c.pop("batch_per_gpu")
        c["shard"] = "heads"
        return c

    def extra(self, world: int, ms_step: float) -> dict:
        ev = self.kernel_events[-min(len(self.kernel_events), 50):]
        torch.cuda.synchronize(self.dev)
        k_ms = float(np.mean([a.elapsed_time(b) for a, b in ev])) if ev else float("nan")
        return {"us_per_layer": round(ms_step * 1e3, 2), "kernel_only_us": round(k_ms * 1e3, 2),
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
    """Samples SM clock and clock-event reasons of one GPU every few ms while
    the timed region runs (NVML; falls back to nvidia-smi when absent)."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, dev: torch.device, period_s: float = 0.005):
        self.dev, self.period = dev, period_s
        self.samples = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._nvml = None

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

            def run():
                while not self._stop.is_set():
                    try:
                        mhz = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                        rs = int(get_reasons(h)) if get_reasons else 0
                        self.samples.append((mhz, rs))
                    except Exception:
                        pass
                    self._stop.wait(self.period)

            self._thread = threading.Thread(target=run, daemon=True)
            self._thread.start()
        except Exception as exc:  # pragma: no cover - NVML missing
            log(f"clock sampling unavailable: {exc}")
        return self

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
# CPU baseline: the oracle port (numpy / BLAS) on a bounded sample
# --------------------------------------------------------------------------
def cpu_slices(cfg: dict, count: int, seed: int = 0):
    """`count` random (batch, q-head) slices of a workload, generated on the
    host with the workload's shapes and distributions: (q [N, D], k, v
    [P_b + N, D], mask [N, P_b + N], kv rows) in float32."""
    from oracle import gorgon_oracle as O
    rng = np.random.default_rng(seed)
    prng = random.Random(seed)
    N, D = cfg["N"], cfg["D"]
    s = 1.0 / math.sqrt(D)
    for _ in range(count):
        P = prng.randint(*cfg["P"]) if isinstance(cfg["P"], tuple) else cfg["P"]
        par = make_tree(cfg, prng)
        q = (rng.standard_normal((N, D), dtype=np.float32) * s)
        k = (rng.standard_normal((P + N, D), dtype=np.float32) * s)
        v = (rng.standard_normal((P + N, D), dtype=np.float32) * s)
        yield q, k, v, O.prefix_tree_mask(par, P, cfg["max_depth"]), P + N


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


def mean_kv_rows(cfg: dict) -> float:
    if isinstance(cfg["P"], tuple):
        return (cfg["P"][0] + cfg["P"][1]) / 2 + cfg["N"]
    return cfg["P"] + cfg["N"]


def cpu_baseline(wl: "Workload", budget_s: float = 12.0, max_slices: int = 64):
    """Times the oracle's tree_attention on (batch, query-head) slices of the
    workload for about `budget_s` seconds and extrapolates to the full layer
    by key/value rows."""
    from oracle import gorgon_oracle as O
    cfg = wl.cfg
    cores = blas_threads()
    total_slices = cfg["B"] * cfg["Hq"]
    times, rows = [], 0
    t_start = time.perf_counter()
    for q, k, v, m, L in cpu_slices(cfg, max_slices, seed=1):
        t0 = time.perf_counter()
        O.tree_attention(q, k, v, m)
        times.append(time.perf_counter() - t0)
        rows += L
        if time.perf_counter() - t_start > budget_s:
            break
    layer_s = sum(times) / rows * (sum(p + cfg["N"] for p in wl.prefixes) / cfg["B"]) * total_slices
    return {
        "value": round(wl.bytes / layer_s / 1e9, 4),
        "unit": "GB/s",
        "cores": cores,
        "kind": "port",
        "us_per_layer": round(layer_s * 1e6, 1),
        "sample": (f"{len(times)} of {total_slices} (batch, q-head) slices of this workload, "
                   f"oracle tree_attention in fp32 numpy/BLAS on {cores} threads, "
                   f"extrapolated by kv rows to the full layer"),
    }


# --------------------------------------------------------------------------
# timing
# --------------------------------------------------------------------------
def dist_setup():
    env = sharding.dist_env()
    return env.world, env.rank, env.local_rank


def time_device(wl: Workload, steps: int, warmup: int, world: int):
    """(ms of the timed steps, mean ms per step, clock summary).  A workload
    whose inputs fit in L2 sets ``flush_l2``: a 256 MB write then evicts L2
    before every step, outside the step's events, and the time is the sum of
    the steps' own event times."""
    dev = wl.dev
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev) if getattr(wl, "flush_l2", False) else None
    for _ in range(warmup):
        wl.step()
    torch.cuda.synchronize(dev)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(dev)
    st = torch.cuda.current_stream(dev)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    with ClockSampler(dev) as clk:
        for i in range(steps):
            if flush is not None:
                flush.fill_(i & 0xff)
            starts[i].record(st)
            wl.step()
            ends[i].record(st)
        torch.cuda.synchronize(dev)
    total_ms = starts[0].elapsed_time(ends[-1])
    per = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    if flush is not None:
        total_ms = float(np.sum(per))
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
    kw = wl.kwargs()

    def one(i):
        k = i % nbuf
        q_d, kt_d, vt_d, par_d = bufs[k]
        with torch.cuda.stream(s_in):
            if i >= nbuf:
                s_in.wait_event(in_free[k])  # step i - 2 has read this buffer set
            q_d.copy_(q_h, non_blocking=True)
            in_ready[k].record(s_in)
        with torch.cuda.stream(s_in2):
            if i >= nbuf:
                s_in2.wait_event(in_free[k])
            kt_d.copy_(kt_h, non_blocking=True)
            vt_d.copy_(vt_h, non_blocking=True)
            par_d.copy_(par_h, non_blocking=True)
            in_ready2[k].record(s_in2)
        s_c.wait_event(in_ready[k])
        s_c.wait_event(in_ready2[k])
        if wl.ragged:
            wl.k[rows] = kt_d
            wl.v[rows] = vt_d
        else:
            wl.k[:, :, P:P + N].copy_(kt_d)
            wl.v[:, :, P:P + N].copy_(vt_d)
        o = G.fused_tree_verify(q_d, wl.k, wl.v, **dict(kw, parents=par_d))
        if post is not None:
            o = post(o)
        in_free[k].record(s_c)
        done[k].record(s_c)
        with torch.cuda.stream(s_out):
            s_out.wait_event(done[k])
            outs_h[k].copy_(o, non_blocking=True)
            o.record_stream(s_out)

    def run(n):
        for i in range(n):
            one(i)
        s_c.wait_stream(s_in)
        s_c.wait_stream(s_in2)
        s_c.wait_stream(s_out)

    run(warmup)
    torch.cuda.synchronize(dev)
    if world > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s_c)
    s_in.wait_event(e0)
    s_in2.wait_event(e0)
    s_out.wait_event(e0)
    run(steps)
    e1.record(s_c)
    torch.cuda.synchronize(dev)
    return e0.elapsed_time(e1), h2d, d2h


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
    # NCCL's version banner goes to stdout, where rank 0's JSON line must be alone
    os.environ["NCCL_DEBUG"] = "WARN"
    sharding.init(sharding.dist_env(), "nccl", dev, timeout_s=120)
    G.load_library()
    # weak scaling by sequence: rank r verifies global sequences [r*B, (r+1)*B)
    if args.shard == "heads":
        if WORKLOADS[args.workload].get("kind", "attn") != "attn":
            raise SystemExit("--shard heads applies to the attention workloads")
        wl = HeadShardWorkload(args.workload, dev, rank, world)
    else:
        wl = make_workload(args.workload, dev, first_seq=rank * WORKLOADS[args.workload]["B"])
    plan = wl.plan()
    total_ms, launch_ms, clocks = time_device(wl, args.steps, args.warmup, world)
    total_ms = max_over_ranks(total_ms, world, dev)
    launch_ms = max_over_ranks(launch_ms, world, dev)
    e2e_steps = args.e2e_steps or args.steps
    e2e_ms, h2d, d2h, e2e_note = wl.e2e(e2e_steps, args.warmup, world)
    e2e_ms = max_over_ranks(e2e_ms, world, dev)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank != 0:
        return
    ms_step = total_ms / args.steps
    value = world * wl.bytes * args.steps / (total_ms * 1e-3) / 1e9
    e2e_val = world * wl.bytes * e2e_steps / (e2e_ms * 1e-3) / 1e9
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
    roof.update({"traffic": NCU_TRAFFIC_BYTES.get((wl.name, plan["backend"])),
                 "launch_us": round(launch_ms * 1e3, 3), "algorithmic_bytes": wl.bytes})
    out = {
        "metric": wl.metric,
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 5),
        "higher_is_better": True,
        "scaling": getattr(wl, "scaling", "weak"),
        "vs_baseline": None,
        "dtype": wl.cfg["dtype"],
        "data": wl.data,
        "config": wl.config(world, plan),
        "pct_of_8tbs": round(100.0 * value / world / 8000.0, 2),
        "roofline": roof,
        "e2e": {
            "value": round(e2e_val, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms / e2e_steps, 5), "note": e2e_note,
        },
        "gpu_launches": plan["launches"] * args.steps,
        "clocks": clocks,
    }
    out.update(wl.extra(world, ms_step))
    if world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = wl.cpu_baseline(args.cpu_budget)
    print(json.dumps(out), flush=True)


def run_reference(args):
    """CPU oracle port on the host cores, same metric and workload.  Each step
    is one (batch, q-head) slice; the layer time is extrapolated by kv rows."""
    world, rank, _ = dist_setup()
    if rank != 0:
        return
    use_all_host_threads()
    from oracle import gorgon_oracle as O
    cfg = WORKLOADS[args.workload]
    if cfg.get("kind", "attn") != "attn":
        run_reference_other(args, cfg, world)
        return
    cores = blas_threads()
    inputs = list(cpu_slices(cfg, 8, seed=0))
    total_slices = cfg["B"] * cfg["Hq"]
    esz = 2 if cfg["dtype"] == "bf16" else 4
    rows = mean_kv_rows(cfg)
    layer_bytes = (2 * rows * cfg["B"] * cfg["Hkv"] * cfg["D"] * esz
                   + 2 * cfg["B"] * cfg["Hq"] * cfg["N"] * cfg["D"] * esz + cfg["B"] * cfg["N"] * 4)
    for i in range(args.warmup):
        O.tree_attention(*inputs[i % len(inputs)][:4])
    t_layer = []
    for i in range(args.steps):
        q, k, v, m, L = inputs[i % len(inputs)]
        t0 = time.perf_counter()
        O.tree_attention(q, k, v, m)
        t_layer.append((time.perf_counter() - t0) / L * rows * total_slices)
    layer_s = float(np.mean(t_layer))
    value = layer_bytes / layer_s / 1e9
    out = {
        "impl": "reference",
        "metric": "tree-verify HBM GB/s (algorithmic bytes / step time)",
        "value": round(value, 4), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(layer_s * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": cfg["dtype"], "data": "synthetic",
        "config": {"workload": args.workload, "batch_per_gpu": cfg["B"], "heads_q": cfg["Hq"],
                   "heads_kv": cfg["Hkv"], "head_dim": cfg["D"],
                   "prefix": list(cfg["P"]) if isinstance(cfg["P"], tuple) else cfg["P"],
                   "tree_nodes": cfg["N"]},
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": "each step one (batch, q-head) slice of the workload through the "
                                   "oracle's tree_attention (fp32 numpy/BLAS), extrapolated by kv "
                                   "rows to the full layer"},
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
    ap.add_argument("--e2e-steps", type=int, default=0, help="steps of the e2e loop (default: --steps)")
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD, choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--shard", default="sequences", choices=["sequences", "heads"],
                    help="multi-GPU split: whole sequences per rank (weak scaling, default) or one layer's "
                         "kv heads per rank with an NCCL all-gather of the output (strong scaling)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
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
