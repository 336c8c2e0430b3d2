"""Spreading tree verification over the GPUs of one node.

Two ways to split the work, one process per GPU:

* by sequence (:func:`shard_range`, :func:`shard_by_weight`): sequences are
  independent (each has its own prefix cache, tree and logits), so every rank
  verifies its own contiguous run of sequences and nothing crosses NVLink on
  the data path; :func:`gather_batch` is there for callers that want every
  rank to hold every output;
* by kv head (:func:`shard_heads`), for one layer that should finish sooner
  on several GPUs: rank r keeps the key/value cache of its kv heads (and the
  query heads that read them), computes their outputs, and
  :func:`gather_heads` all-gathers the head slices into the layer's output.

``torch.distributed`` (NCCL on GPUs, gloo on CPU) carries barriers, the
max-over-ranks timing and the gathers.
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass
from typing import List, Sequence, Tuple

import torch
import torch.distributed as dist

__all__ = ["DistEnv", "dist_env", "init", "shard_range", "shard_by_weight", "shard_heads", "max_over_ranks",
           "gather_batch", "gather_heads"]


@dataclass(frozen=True)
class DistEnv:
    rank: int
    world: int
    local_rank: int


def dist_env() -> DistEnv:
    """Rank layout from the launcher's environment (torchrun sets these)."""
    return DistEnv(int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
                   int(os.environ.get("LOCAL_RANK", "0")))


def init(env: DistEnv, backend: str, device: torch.device = None, timeout_s: int = 120) -> None:
    """Joins the process group (a no-op for one rank).  The short timeout makes
    ranks that wait on a missing peer fail instead of hanging."""
    if env.world <= 1 or dist.is_initialized():
        return
    kw = dict(timeout=datetime.timedelta(seconds=timeout_s))
    if device is not None and device.type == "cuda":
        kw["device_id"] = device
    dist.init_process_group(backend, rank=env.rank, world_size=env.world, **kw)


def shard_range(n_items: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous [start, end) share of n_items for `rank`; sizes differ by at most one."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    return rank * n_items // world, (rank + 1) * n_items // world


def shard_by_weight(weights: Sequence[int], world: int, rank: int) -> Tuple[int, int]:
    """Contiguous [start, end) run of items for `rank` that splits the total
    weight (e.g. key/value rows of ragged sequences) as evenly as contiguous
    runs allow: rank r starts at the first item whose prefix weight reaches
    r / world of the total."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    total = sum(weights)
    bounds: List[int] = [0]
    acc = 0
    k = 1
    for i, w in enumerate(weights):
        acc += w
        while k < world and acc * world >= k * total:
            bounds.append(i + 1)
            k += 1
    while len(bounds) < world:
        bounds.append(len(weights))
    bounds.append(len(weights))
    return bounds[rank], bounds[rank + 1]


def shard_heads(heads_kv: int, heads_q: int, world: int, rank: int) -> Tuple[Tuple[int, int], Tuple[int, int]]:
    """This rank's kv heads [h0, h1) and the query heads that read them,
    [h0 * g, h1 * g) with g = heads_q / heads_kv.  Every rank gets the same
    number of heads, so the output gather moves equal slices."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    if heads_kv % world or heads_q % heads_kv:
        raise ValueError(f"{heads_kv} kv heads ({heads_q} query heads) do not split evenly over {world} ranks")
    per = heads_kv // world
    g = heads_q // heads_kv
    return (rank * per, (rank + 1) * per), (rank * per * g, (rank + 1) * per * g)


def gather_heads(local: torch.Tensor, out: torch.Tensor = None) -> torch.Tensor:
    """All-gathers every rank's head slice [B, h, ...] into [B, world * h, ...]
    (rank r's slice at heads r*h .. r*h + h): one all-gather of the equally
    sized slices, then one copy into the batch-major layout.  With one rank
    the slice is the whole output and is returned as it is."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return local
    world = dist.get_world_size()
    B, h = local.shape[0], local.shape[1]
    rest = tuple(local.shape[2:])
    flat = torch.empty((world,) + tuple(local.shape), dtype=local.dtype, device=local.device)
    if dist.get_backend() == "nccl":
        dist.all_gather_into_tensor(flat.view(-1), local.contiguous().view(-1))
    else:
        dist.all_gather(list(flat.unbind(0)), local.contiguous())
    if out is None:
        out = torch.empty((B, world * h) + rest, dtype=local.dtype, device=local.device)
    out.view((B, world, h) + rest).copy_(flat.movedim(0, 1))
    return out


def max_over_ranks(value: float, device: torch.device = None) -> float:
    """The largest value any rank holds (the job's time is its slowest rank's)."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64,
                     device=device if device is not None else torch.device("cpu"))
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_batch(local: torch.Tensor) -> torch.Tensor:
    """Concatenates every rank's equally sized batch shard along dim 0."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return local
    world = dist.get_world_size()
    if dist.get_backend() == "nccl":
        out = torch.empty((world * local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype,
                          device=local.device)
        dist.all_gather_into_tensor(out, local.contiguous())
        return out
    parts = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(parts, local.contiguous())
    return torch.cat(parts, 0)
