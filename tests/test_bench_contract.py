"""Host logic of bench.py that the JSON line depends on, checked on CPU:
the sequence split covers the batch once at every GPU count, the ranks'
algorithmic bytes add up to the whole job's (so a strong-scaling value is the
job's bytes over the slowest rank's time), ragged batches are split by
key/value rows, and the `config` dict names the split and how the output is
gathered.  The reference arm prints the same dict (attn_config needs no GPU)."""
from __future__ import annotations

import pytest

import bench


ATTN = [n for n, c in bench.WORKLOADS.items() if c.get("kind", "attn") == "attn"]


@pytest.mark.parametrize("name", ["verify-b16-p8192-n64", "ragged-b16-p1k-8k-n64", "verify-b32-p4096-n64"])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_strong_split_covers_the_batch_once(name, world):
    cfg = bench.WORKLOADS[name]
    spans = [bench.seq_shard(name, world, r, "strong") for r in range(world)]
    starts = [s for s, _ in spans]
    assert starts[0] == 0
    assert all(s0 + n0 == s1 for (s0, n0), s1 in zip(spans, starts[1:]))
    assert sum(n for _, n in spans) == cfg["B"]
    # the ranks' bytes add up to the job's bytes
    whole = bench.attn_bytes(cfg, bench.attn_sequences(cfg, 0, cfg["B"])[0])
    parts = [bench.attn_bytes(cfg, bench.attn_sequences(cfg, s, n)[0]) for s, n in spans]
    ragged_extra = 4 * (world - 1) if isinstance(cfg["P"], tuple) else 0  # one cu_seqlens entry more per rank
    assert sum(parts) == whole + ragged_extra


def test_ragged_split_balances_key_value_rows():
    name = "ragged-b16-p1k-8k-n64"
    cfg = bench.WORKLOADS[name]
    prefixes, _ = bench.attn_sequences(cfg, 0, cfg["B"])
    for world in (2, 4, 8):
        loads = []
        for r in range(world):
            s, n = bench.seq_shard(name, world, r, "strong")
            loads.append(sum(p + cfg["N"] for p in prefixes[s:s + n]))
        assert max(loads) - sum(loads) / world <= max(p + cfg["N"] for p in prefixes)


def test_sequences_do_not_depend_on_the_split():
    cfg = bench.WORKLOADS["ragged-b16-p1k-8k-n64"]
    whole_p, whole_t = bench.attn_sequences(cfg, 0, cfg["B"])
    part_p, part_t = bench.attn_sequences(cfg, 5, 4)
    assert part_p == whole_p[5:9] and part_t == whole_t[5:9]


@pytest.mark.parametrize("name", ATTN)
def test_config_names_the_workload_and_split(name):
    cfg = bench.WORKLOADS[name]
    one = bench.attn_config(name, 1, "strong")
    assert one["workload"] == name and one["parallelism"] == "single GPU" and one["batch"] == cfg["B"]
    if cfg["B"] >= 8:
        eight = bench.attn_config(name, 8, "strong")
        assert "strong scaling" in eight["parallelism"] and "no collective" in eight["parallelism"]
        assert eight["batch"] == cfg["B"]
    weak = bench.attn_config(name, 2, "weak")
    assert weak["batch"] == 2 * cfg["B"] and "weak scaling" in weak["parallelism"]


def test_head_split_config_says_how_the_output_is_gathered():
    fused = bench.attn_config("wide-b8-p32k-n256", 8, "heads", "fused")
    nccl = bench.attn_config("wide-b8-p32k-n256", 8, "heads", "nccl")
    assert "1 of 8 kv heads per GPU" in fused["parallelism"]
    assert "NVLink stores" in fused["parallelism"] and "NCCL" in nccl["parallelism"]
    # 70 MB per GPU fits in L2: that line is timed from a flushed L2
    assert fused["l2"].startswith("L2 flushed")


def test_l2_rule_follows_the_bytes_per_gpu():
    assert bench.attn_config("verify-b16-p8192-n64", 1, "strong")["l2"].startswith("inputs larger than L2")
    assert bench.attn_config("verify-b16-p8192-n64", 8, "strong")["l2"].startswith("L2 flushed")
    assert bench.attn_config("verify-b1-p2048-n64", 1, "strong")["l2"].startswith("L2 flushed")
