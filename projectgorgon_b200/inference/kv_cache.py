"""KV-cache trim-on-reject on the GPU.

``apply_cache_slice`` keeps the reference's contract
(``src/gorgon/inference/kv_cache.py:89-108``): copies of ``keys``/``values``
with ``new[:L] = old[idx]`` along dim 0.  ``GorgonKVCache`` keeps the
reference's class API (``kv_cache.py:21-86``) and adds ``trim``, which compacts
the accepted tree rows of every layer into contiguous slots in one launch,
in place, from device-side indices (no host sync).
"""
from __future__ import annotations

import math
from typing import List, Optional, Sequence, Tuple, Union

import torch

from .. import _abi
from .._util import on_device, require_cuda, stream_ptr

PastKV = Tuple[Tuple[torch.Tensor, torch.Tensor], ...]


def _launch_trim(k_src: List[torch.Tensor], v_src: List[torch.Tensor],
                 k_dst: Optional[List[torch.Tensor]], v_dst: Optional[List[torch.Tensor]],
                 batch: int, heads: int, seq: int, head_dim: int, strides: Tuple[int, int, int],
                 elem_bytes: int, idx: torch.Tensor, lens: torch.Tensor,
                 dst_start: Optional[torch.Tensor]) -> None:
    p = _abi.KvTrimParams()
    p.elem_bytes = elem_bytes
    p.layers, p.batch, p.heads, p.seq_capacity, p.head_dim = len(k_src), batch, heads, seq, head_dim
    p.stride_b, p.stride_h, p.stride_s = strides
    arrays = [_abi.pointer_array([t.data_ptr() for t in k_src]),
              _abi.pointer_array([t.data_ptr() for t in v_src])]
    p.k_src, p.v_src = arrays
    if k_dst is not None:
        arrays += [_abi.pointer_array([t.data_ptr() for t in k_dst]),
                   _abi.pointer_array([t.data_ptr() for t in v_dst])]
        p.k_dst, p.v_dst = arrays[2], arrays[3]
    _run_trim(p, k_src[0].device, idx, lens, dst_start)


def _run_trim(p, dev: torch.device, idx: torch.Tensor, lens: torch.Tensor,
              dst_start: Optional[torch.Tensor]) -> None:
    """Fills the per-call fields of a prepared parameter block and launches."""
    p.src_idx, p.idx_stride_b, p.max_len = idx.data_ptr(), idx.stride(0), idx.shape[1]
    p.lens = lens.data_ptr()
    p.dst_start = dst_start.data_ptr() if dst_start is not None else 0
    with on_device(dev):
        _abi.check(_abi.lib().gorgon_kv_trim(p, stream_ptr(dev)), "gorgon_kv_trim")


def apply_cache_slice(keys: torch.Tensor, values: torch.Tensor,
                      accepted_indices: Union[Sequence[int], torch.Tensor]
                      ) -> Tuple[torch.Tensor, torch.Tensor, int]:
    """Copy accepted KV entries to the front of the cache.

    Returns ``(new_keys, new_values, new_length)``; the inputs are not
    modified.  Rows are taken along dim 0, any trailing shape."""
    require_cuda("keys and values", keys, values)
    if keys.shape[0] != values.shape[0]:
        raise RuntimeError("keys and values must have the same length")
    new_k = keys.clone()
    new_v = values.clone()
    if isinstance(accepted_indices, torch.Tensor):
        idx = accepted_indices.to(device=keys.device, dtype=torch.int32).reshape(1, -1).contiguous()
    else:
        idx = torch.tensor([list(accepted_indices)], dtype=torch.int32, device=keys.device)
    L = idx.shape[1]
    if L == 0:
        return new_k, new_v, 0
    if L > keys.shape[0]:
        raise RuntimeError("more accepted indices than cache rows")
    kc, vc = keys.contiguous(), values.contiguous()
    if kc.dtype != vc.dtype or kc[0].numel() != vc[0].numel():
        # K and V rows differ in type or width: trim them as two calls
        apply = [(kc, new_k), (vc, new_v)]
    else:
        apply = [(kc, new_k, vc, new_v)]
    lens = torch.tensor([L], dtype=torch.int32, device=keys.device)
    for item in apply:
        if len(item) == 2:
            src, dst = item
            srcs, dsts, vsrc, vdst = [src], [dst], [src], [dst]
            ref = src
        else:
            srcs, dsts, vsrc, vdst = [item[0]], [item[1]], [item[2]], [item[3]]
            ref = item[0]
        row = max(1, int(math.prod(ref.shape[1:])))
        seq = ref.shape[0]
        _launch_trim(srcs, vsrc, dsts, vdst, 1, 1, seq, row, (seq * row, seq * row, row),
                     ref.element_size(), idx, lens, None)
    return new_k, new_v, L


class GorgonKVCache:
    """Per-layer ``(K, V)`` cache in HF layout ``[batch, heads, seq, head_dim]``.

    ``update``/``checkpoint``/``rollback``/``trim_to``/``clear`` behave as the
    reference's (``src/gorgon/inference/kv_cache.py:21-86``).  ``trim`` is the
    trim-on-reject gather of the accepted tree path, all layers at once.
    """

    def __init__(self) -> None:
        self._cache: Optional[PastKV] = None
        self._checkpoint: Optional[PastKV] = None
        self._seq_len: int = 0
        self._trim_plan = None   # validated layout + per-layer pointer arrays of the current cache
        self._dst_fill = {}      # (batch, start) -> device int32 [batch] filled with start

    @property
    def past_key_values(self) -> Optional[PastKV]:
        return self._cache

    @property
    def seq_len(self) -> int:
        return self._seq_len

    def update(self, past_kv: PastKV) -> None:
        self._cache = past_kv
        if past_kv and past_kv[0][0].numel() > 0:
            self._seq_len = past_kv[0][0].shape[2]
        else:
            self._seq_len = 0

    def checkpoint(self) -> None:
        if self._cache is None:
            self._checkpoint = None
            return
        self._checkpoint = tuple((k.clone(), v.clone()) for k, v in self._cache)

    def rollback(self) -> None:
        if self._checkpoint is not None:
            self._cache = self._checkpoint
            self._checkpoint = None
            if self._cache and self._cache[0][0].numel() > 0:
                self._seq_len = self._cache[0][0].shape[2]
            else:
                self._seq_len = 0

    def trim_to(self, length: int) -> None:
        if self._cache is None:
            return
        self._cache = tuple((k[:, :, :length, :], v[:, :, :length, :]) for k, v in self._cache)
        self._seq_len = length

    def clear(self) -> None:
        self._cache = None
        self._checkpoint = None
        self._seq_len = 0

    def trim(self, src_idx: torch.Tensor, lens: torch.Tensor,
             dst_start: Union[torch.Tensor, int, None] = None) -> None:
        """In place, for every layer, batch row b and head h:
        ``cache[b, h, dst_start[b] + r] = cache[b, h, src_idx[b, r]]`` for
        ``r < lens[b]``.  ``src_idx`` int ``[B, max_len]`` and ``lens`` ``[B]``
        may be device tensors straight from the verifier (no host sync);
        ``dst_start`` is ``[B]``, an int, or None for 0."""
        if self._cache is None:
            return
        params = self._prepared_trim()
        k0 = self._cache[0][0]
        dev = k0.device
        B = k0.shape[0]
        idx = src_idx.to(device=dev, dtype=torch.int32)
        if idx.dim() == 1:
            idx = idx.unsqueeze(0)
        idx = idx.contiguous()
        ln = lens.to(device=dev, dtype=torch.int32).reshape(-1).contiguous()
        if idx.shape[0] != B or ln.numel() != B:
            raise RuntimeError("src_idx and lens need one row per batch element")
        if isinstance(dst_start, int):
            ds = self._dst_fill.get((B, dst_start))
            if ds is None or ds.device != dev:
                ds = torch.full((B,), dst_start, dtype=torch.int32, device=dev)
                self._dst_fill[(B, dst_start)] = ds
        elif dst_start is None:
            ds = None
        else:
            ds = dst_start.to(device=dev, dtype=torch.int32).reshape(-1).contiguous()
        _run_trim(params, dev, idx, ln, ds)

    def _prepared_trim(self):
        """The trim's parameter block for the current layers: the layout is
        checked and the per-layer pointer arrays built once per cache (the
        cache tuple is replaced, never mutated, by update/rollback/trim_to)."""
        c = self._cache
        plan = self._trim_plan
        if plan is not None and plan[0] is c and plan[1] == c[0][0].data_ptr():
            return plan[2]
        k0 = c[0][0]
        require_cuda("cache tensors", k0)
        B, H, S, D = k0.shape
        for k, v in c:
            if k.shape != k0.shape or v.shape != k0.shape or k.dtype != k0.dtype or v.dtype != k0.dtype:
                raise RuntimeError("all layers must share one shape and dtype")
            if k.stride() != k0.stride() or v.stride() != k0.stride() or k.stride(-1) != 1:
                raise RuntimeError("all layers must share one stride layout with head_dim contiguous")
            if k.device != k0.device or v.device != k0.device:
                raise RuntimeError("all layers must be on one device")
        p = _abi.KvTrimParams()
        p.elem_bytes = k0.element_size()
        p.layers, p.batch, p.heads, p.seq_capacity, p.head_dim = len(c), B, H, S, D
        p.stride_b, p.stride_h, p.stride_s = k0.stride(0), k0.stride(1), k0.stride(2)
        arrays = (_abi.pointer_array([k.data_ptr() for k, _ in c]),
                  _abi.pointer_array([v.data_ptr() for _, v in c]))
        p.k_src, p.v_src = arrays
        self._trim_plan = (c, k0.data_ptr(), p, arrays)   # the arrays stay alive with the block
        return p
