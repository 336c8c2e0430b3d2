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

import ctypes
import datetime
import os
from dataclasses import dataclass
from typing import List, Sequence, Tuple

import torch
import torch.distributed as dist

__all__ = ["DistEnv", "dist_env", "init", "shard_range", "shard_by_weight", "shard_heads", "max_over_ranks",
           "sum_over_ranks", "gather_batch", "gather_heads", "head_sharded_output", "gather_heads_inplace"]


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


def head_sharded_output(batch: int, heads_q: int, n: int, d: int, dtype: torch.dtype, device: torch.device,
                        world: int, rank: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """(full, local): the layer output held head-major -- a ``[Hq, B, N, D]``
    buffer, so the query heads of rank r are one contiguous chunk -- and this
    rank's ``[B, Hq / world, N, D]`` view of its own chunk, for the attention
    to write straight into (``tree_attention(..., out=local)``).
    :func:`gather_heads_inplace` then assembles the layer with one all-gather
    and no re-layout copy."""
    if world < 1 or not 0 <= rank < world or heads_q % world:
        raise ValueError(f"{heads_q} query heads do not split evenly over {world} ranks")
    per = heads_q // world
    full = torch.empty((heads_q, batch, n, d), dtype=dtype, device=device)
    return full, full[rank * per:(rank + 1) * per].permute(1, 0, 2, 3)


def gather_heads_inplace(full: torch.Tensor, async_op: bool = False):
    """All-gathers a head-major output (:func:`head_sharded_output`) in place:
    rank r's chunk is the send buffer and the whole buffer the receive buffer
    (NCCL's in-place all-gather), so every rank ends with the layer's output.
    Returns it as ``[B, Hq, N, D]`` (a view with head-major strides); with
    ``async_op`` returns ``(view, work)``, the gather running on NCCL's stream
    once the work queued so far on the current stream is done, so the caller
    can queue more compute before ``work.wait()``."""
    work = None
    if dist.is_initialized() and dist.get_world_size() > 1:
        world, rank = dist.get_world_size(), dist.get_rank()
        flat = full.view(-1)
        chunk = flat.numel() // world
        mine = flat[rank * chunk:(rank + 1) * chunk]
        if dist.get_backend() == "nccl":
            work = dist.all_gather_into_tensor(flat, mine, async_op=async_op)
        else:
            work = dist.all_gather(list(flat.view(world, chunk).unbind(0)), mine.clone(), async_op=async_op)
    view = full.permute(1, 0, 2, 3)
    return (view, work) if async_op else view


class _DeviceArray:
    """A raw device allocation described by the CUDA array interface (so
    torch can view it without owning it)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": (nbytes,), "typestr": "|u1",
                                         "version": 3, "strides": None}


class PeerHeadOutput:
    """The head-major layer output ``[Hq, B, N, D]`` of a layer split by kv
    head, with the gather fused into the attention kernel.

    Every rank allocates its buffer with ``gorgon_peer_buffer_alloc``, the
    handles go round the process group (any backend; only bytes on the host),
    and each rank maps the others' buffers (CUDA IPC; the kernels reach them
    over NVLink).  ``tree_attention(..., out=self.local, peer_group=self)``
    then writes this rank's query heads into every rank's buffer from the
    kernel's epilogue and waits on the stream for the other ranks' heads: no
    all-gather call, the transfer overlapping the attention tile by tile.
    ``full`` is this rank's buffer as ``[B, Hq, N, D]`` (head-major strides),
    ``local`` the ``[B, Hq / world, N, D]`` part this rank computes.  Call
    :meth:`close` on every rank (it synchronises them) before the process
    group goes."""

    SIGNAL_BYTES = 256  # four uint64 signal words, padded

    def __init__(self, batch: int, heads_q: int, heads_kv: int, n: int, d: int, dtype: torch.dtype,
                 device: torch.device, world: int, rank: int, group=None):
        from . import _abi
        (_, _), (q0, q1) = shard_heads(heads_kv, heads_q, world, rank)
        if q1 - q0 != heads_q // world:
            raise ValueError(f"{heads_q} query heads do not split evenly over {world} ranks")
        self.world, self.rank, self.group = world, rank, group
        esz = torch.tensor([], dtype=dtype).element_size()
        data = heads_q * batch * n * d * esz
        self.signal_offset = (data + 255) // 256 * 256
        nbytes = self.signal_offset + self.SIGNAL_BYTES
        lib = _abi.lib()
        own, handle = ctypes.c_void_p(), _abi.IpcHandle()
        with torch.cuda.device(device):
            _abi.check(lib.gorgon_peer_buffer_alloc(nbytes, ctypes.byref(own), ctypes.byref(handle)),
                       "gorgon_peer_buffer_alloc")
            self._own = own.value
            self._opened: List[int] = []
            handles = [bytes(handle.bytes)]
            if world > 1:
                handles = [None] * world
                dist.all_gather_object(handles, bytes(handle.bytes), group=group)
            bases = []
            for r in range(world):
                if r == rank:
                    bases.append(self._own)
                    continue
                h = _abi.IpcHandle()
                ctypes.memmove(h.bytes, handles[r], 64)
                p = ctypes.c_void_p()
                _abi.check(lib.gorgon_peer_buffer_open(ctypes.byref(h), ctypes.byref(p)), "gorgon_peer_buffer_open")
                self._opened.append(p.value)
                bases.append(p.value)
        base_arr = (ctypes.c_void_p * _abi.MAX_PEERS)(*bases)
        self._group = _abi.PeerGroup(world, rank, base_arr, self.signal_offset)
        raw = torch.as_tensor(_DeviceArray(self._own, nbytes), device=device)
        self._raw = raw
        self.full_head_major = raw[:data].view(dtype).view(heads_q, batch, n, d)
        self.full = self.full_head_major.permute(1, 0, 2, 3)
        self.local = self.full_head_major[q0:q1].permute(1, 0, 2, 3)

    def group_ref(self):
        return ctypes.byref(self._group)

    def close(self) -> None:
        """Unmaps the other ranks' buffers and frees this rank's, after every
        rank has stopped using them (a barrier on the group)."""
        from . import _abi
        if self._own is None:
            return
        lib = _abi.lib()
        torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier(group=self.group)
        for p in self._opened:
            lib.gorgon_peer_buffer_close(ctypes.c_void_p(p))
        self._opened = []
        if self.world > 1:
            dist.barrier(group=self.group)
        self._raw = self.full_head_major = self.full = self.local = None
        lib.gorgon_peer_buffer_free(ctypes.c_void_p(self._own))
        self._own = None


def max_over_ranks(value: float, device: torch.device = None) -> float:
    """The largest value any rank holds (the job's time is its slowest rank's)."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64,
                     device=device if device is not None else torch.device("cpu"))
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value: float, device: torch.device = None) -> float:
    """The sum of every rank's value (e.g. the bytes of the whole job)."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64,
                     device=device if device is not None else torch.device("cpu"))
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def gather_batch(local: torch.Tensor) -> torch.Tensor:
    """Concatenates every rank's batch shard along dim 0, in rank order.

    Shards may differ in length (``shard_range`` and ``shard_by_weight`` give
    uneven runs when the batch does not divide): the ranks first exchange
    their lengths, every shard is padded to the longest for one equal-sized
    all-gather, and the padding is dropped.  The trailing dimensions must
    agree on every rank."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return local
    world = dist.get_world_size()
    nccl = dist.get_backend() == "nccl"
    dev = local.device if nccl else torch.device("cpu")
    lens = torch.zeros(world, dtype=torch.int64, device=dev)
    mine = torch.tensor([local.shape[0]], dtype=torch.int64, device=dev)
    if nccl:
        dist.all_gather_into_tensor(lens, mine)
    else:
        dist.all_gather(list(lens.unbind(0)), mine[0].clone())
    sizes = [int(x) for x in lens.cpu().tolist()]
    most = max(sizes)
    rest = tuple(local.shape[1:])
    padded = local.contiguous()
    if local.shape[0] < most:
        padded = torch.cat([padded, padded.new_zeros((most - local.shape[0],) + rest)], 0)
    if nccl:
        allp = torch.empty((world * most,) + rest, dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(allp, padded)
        parts = list(allp.split(most, 0))
    else:
        parts = [torch.empty_like(padded) for _ in range(world)]
        dist.all_gather(parts, padded)
    if all(n == most for n in sizes):
        return torch.cat(parts, 0)
    return torch.cat([p[:n] for p, n in zip(parts, sizes)], 0)
