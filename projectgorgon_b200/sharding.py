"""Spreading tree verification over the GPUs of one node.

The verify path shards without any data exchange: sequences are independent
(each has its own prefix cache, tree and logits), so every rank verifies its
own contiguous run of sequences and nothing crosses NVLink on the data path.
One process drives one GPU; ``torch.distributed`` (NCCL on GPUs, gloo on CPU)
is only used for barriers, the max-over-ranks timing and, where a caller
wants every rank to hold every sequence's output, :func:`gather_batch`.
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass
from typing import List, Sequence, Tuple

import torch
import torch.distributed as dist

__all__ = ["DistEnv", "dist_env", "init", "shard_range", "shard_by_weight", "max_over_ranks",
           "gather_batch"]


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
