"""Tree attention over ``[prefix | tree]`` key/value rows on B200.

``tree_attention`` is the one entry every reference-named wrapper routes to.
It keeps the reference's 2-D call form ``tree_attention(q, k, v, mask)`` with
``q [N, D]``, ``k, v [M, D]``, ``mask [N, M]`` (``tree_attention_ref``,
``src/gorgon/kernels/tree_attention_ref.py:8-18``) and adds:

* a key/value prefix: ``k, v [P + N, D]`` with a tree-only mask ``[N, N]``
  (prefix rows are visible to every tree row) or a full ``[N, P + N]`` mask;
* heads and grouped-query attention: ``q [B, Hq, N, D]``, ``k, v [B, Hkv, L, D]``,
  query head ``h`` reading kv head ``h // (Hq // Hkv)``;
* the mask-free form: ``parents=`` instead of a mask, walked ``max_depth`` hops
  in the kernel (``fused_tree_verify_triton.py:52-63``);
* ragged batches: ``k, v [total, Hkv, D]`` plus ``cu_seqlens int32 [B + 1]``.

All work runs in ``libgorgon_b200.so``; host tensors raise ``ValueError``.
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional, Sequence, Tuple, Union

import torch

from .. import _abi
from .._util import gorgon_dtype, on_device, parents_tensor, ptr, require_cuda, stream_ptr, workspace

_BACKENDS = {"auto": _abi.BACKEND_AUTO, "simt": _abi.BACKEND_SIMT, "tcgen05": _abi.BACKEND_TCGEN05,
             "tcgen05-pair": _abi.BACKEND_TCGEN05_PAIR, "tcgen05-cta": _abi.BACKEND_TCGEN05_CTA}


def _as4(x: torch.Tensor, name: str) -> torch.Tensor:
    if x.dim() == 2:
        return x.unsqueeze(0).unsqueeze(0)
    if x.dim() == 3:
        return x.unsqueeze(0)
    if x.dim() == 4:
        return x
    raise RuntimeError(f"{name} must be 2-D, 3-D or 4-D, got {tuple(x.shape)}")


def _last_contig(x: torch.Tensor) -> torch.Tensor:
    return x if x.stride(-1) == 1 else x.contiguous()


def tree_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    tree_mask: Optional[torch.Tensor] = None,
    *,
    parents: Union[Sequence[int], torch.Tensor, None] = None,
    max_depth: Optional[int] = None,
    cu_seqlens: Optional[torch.Tensor] = None,
    max_seqlen: Optional[int] = None,
    scale: Optional[float] = None,
    out_dtype: Optional[torch.dtype] = None,
    return_lse: bool = False,
    backend: str = "auto",
    num_splits: int = 0,
    out: Optional[torch.Tensor] = None,
    peer_group=None,
) -> Union[torch.Tensor, Tuple[torch.Tensor, torch.Tensor]]:
    """Masked softmax attention of tree queries over prefix + tree keys.

    Exactly one of ``tree_mask`` and ``parents`` is given.  Returns ``out``
    shaped like ``q`` (dtype ``out_dtype`` or ``q.dtype``), and with
    ``return_lse`` also the natural-log sum-exp ``[B, Hq, N]`` (float32).
    ``out``, when given, is written instead of a new tensor: 4-D ``q`` only,
    shape ``[B, Hq, N, D]``, any strides with ``head_dim`` contiguous (e.g. a
    head-major slice of a larger buffer).  ``peer_group`` (a
    ``sharding.PeerHeadOutput``, with ``out`` its ``local`` view) also writes
    the rows into every other rank's copy of the buffer from the kernel's
    epilogue and waits on the stream until the other ranks' rows have landed
    here (``gorgon_tree_attn_gather``).
    """
    prep = _prepare(q, k, v, tree_mask, parents, max_depth, cu_seqlens, max_seqlen, scale,
                    out_dtype, return_lse, backend, num_splits, out)
    lib = _abi.lib()
    dev = prep.out.device
    with on_device(dev):
        nbytes = lib.gorgon_tree_attn_workspace_size(prep.p)
        ws = workspace(nbytes, dev) if nbytes else None
        if peer_group is None:
            _abi.check(lib.gorgon_tree_attn(prep.p, ptr(ws), nbytes, stream_ptr(dev)), "gorgon_tree_attn")
        else:
            _abi.check(lib.gorgon_tree_attn_gather(prep.p, peer_group.group_ref(), ptr(ws), nbytes,
                                                   stream_ptr(dev)), "gorgon_tree_attn_gather")
    out = prep.out
    if q.dim() != 4:
        out = out.reshape(tuple(q.shape[:-1]) + (out.shape[-1],))
    if return_lse:
        return out, prep.lse
    return out


def tree_attention_plan(q, k, v, tree_mask=None, **kwargs) -> dict:
    """The launch plan ``tree_attention`` would use for these arguments:
    ``backend`` ("simt", "tcgen05" for the single-CTA tensor-core kernel or
    "tcgen05-pair" for the CTA-pair one), ``splits`` (CTAs of the tensor-core
    grid, or the CUDA-core kernel's key splits), ``launches`` (kernels per
    call) and ``workspace_bytes``.  ``backend=`` in the arguments requests one
    ("auto", "simt", "tcgen05" -- either tensor-core shape, the planner's
    pick -- "tcgen05-pair" or "tcgen05-cta")."""
    args = dict(parents=None, max_depth=None, cu_seqlens=None, max_seqlen=None, scale=None,
                out_dtype=None, return_lse=False, backend="auto", num_splits=0)
    args.update(kwargs)
    prep = _prepare(q, k, v, tree_mask, args["parents"], args["max_depth"], args["cu_seqlens"],
                    args["max_seqlen"], args["scale"], args["out_dtype"], args["return_lse"],
                    args["backend"], args["num_splits"])
    lib = _abi.lib()
    be, sp, ln = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
    with on_device(prep.out.device):
        _abi.check(lib.gorgon_tree_attn_plan(prep.p, ctypes.byref(be), ctypes.byref(sp), ctypes.byref(ln)),
                   "gorgon_tree_attn_plan")
        nbytes = lib.gorgon_tree_attn_workspace_size(prep.p)
    names = {_abi.BACKEND_SIMT: "simt", _abi.BACKEND_TCGEN05: "tcgen05", _abi.BACKEND_TCGEN05_PAIR: "tcgen05-pair"}
    return {"backend": names.get(be.value, str(be.value)), "splits": sp.value, "launches": ln.value,
            "workspace_bytes": int(nbytes)}


class _Prepared:
    __slots__ = ("p", "out", "lse", "keep")

    def __init__(self, p, out, lse, keep):
        self.p, self.out, self.lse, self.keep = p, out, lse, keep


def _prepare(q, k, v, tree_mask, parents, max_depth, cu_seqlens, max_seqlen, scale, out_dtype,
             return_lse, backend, num_splits, out=None) -> _Prepared:
    if (tree_mask is None) == (parents is None):
        raise RuntimeError("pass exactly one of tree_mask and parents")
    tensors = [q, k, v] + ([tree_mask] if tree_mask is not None else [])
    require_cuda("q, k, v" + (" and mask" if tree_mask is not None else ""), *tensors)
    if backend not in _BACKENDS:
        raise RuntimeError(f"backend must be one of {sorted(_BACKENDS)}")
    dev = q.device
    if k.device != dev or v.device != dev:
        raise RuntimeError("q, k, v must be on the same device")
    if not (q.dtype == k.dtype == v.dtype):
        common = torch.promote_types(torch.promote_types(q.dtype, k.dtype), v.dtype)
        q, k, v = q.to(common), k.to(common), v.to(common)
    dt = gorgon_dtype(q.dtype)
    out_dt = out_dtype if out_dtype is not None else (out.dtype if out is not None else q.dtype)
    odt = gorgon_dtype(out_dt)

    q_shape = q.shape
    q4 = _last_contig(_as4(q, "q"))
    B, Hq, N, D = q4.shape
    if cu_seqlens is not None:
        if k.dim() != 3 or v.dim() != 3:
            raise RuntimeError("with cu_seqlens, k and v must be [total, heads_kv, head_dim]")
        k3, v3 = _last_contig(k), _last_contig(v)
        Hkv = k3.shape[1]
        if k3.shape[2] != D or v3.shape != k3.shape:
            raise RuntimeError("k and v must be [total, heads_kv, head_dim] with q's head_dim")
        cu = cu_seqlens.to(device=dev, dtype=torch.int32).contiguous()
        if cu.numel() != B + 1:
            raise RuntimeError("cu_seqlens must have batch + 1 entries")
        L = int(max_seqlen) if max_seqlen is not None else int((cu[1:] - cu[:-1]).max().item())
        ks = (0, k3.stride(1), k3.stride(0))
        vs = (0, v3.stride(1), v3.stride(0))
        kk, vv = k3, v3
    else:
        cu = None
        k4, v4 = _last_contig(_as4(k, "k")), _last_contig(_as4(v, "v"))
        if k4.shape[0] != B or v4.shape != k4.shape or k4.shape[3] != D:
            raise RuntimeError(f"k/v shape {tuple(k.shape)} does not match q {tuple(q_shape)}")
        Hkv, L = k4.shape[1], k4.shape[2]
        ks = (k4.stride(0), k4.stride(1), k4.stride(2))
        vs = (v4.stride(0), v4.stride(1), v4.stride(2))
        kk, vv = k4, v4
    if Hkv == 0 or Hq % Hkv != 0:
        raise RuntimeError(f"heads_q ({Hq}) must be a multiple of heads_kv ({Hkv})")

    if out is None:
        out = torch.empty((B, Hq, N, D), dtype=out_dt, device=dev)
    else:
        if q.dim() != 4 or tuple(out.shape) != (B, Hq, N, D):
            raise RuntimeError(f"out must be [B, Hq, N, D] = {(B, Hq, N, D)} for a 4-D q, got {tuple(out.shape)}")
        if out.dtype != out_dt or out.device != dev or out.stride(-1) != 1:
            raise RuntimeError("out must have the output dtype, q's device and a contiguous last dimension")
    lse = torch.empty((B, Hq, N), dtype=torch.float32, device=dev) if return_lse else None
    p = _abi.TreeAttnParams()
    p.dtype, p.out_dtype = dt, odt
    p.batch, p.heads_q, p.heads_kv, p.n_tree, p.kv_len, p.head_dim = B, Hq, Hkv, N, L, D
    p.q, p.q_stride_b, p.q_stride_h, p.q_stride_n = q4.data_ptr(), q4.stride(0), q4.stride(1), q4.stride(2)
    p.k, (p.k_stride_b, p.k_stride_h, p.k_stride_s) = kk.data_ptr(), ks
    p.v, (p.v_stride_b, p.v_stride_h, p.v_stride_s) = vv.data_ptr(), vs
    p.out, p.o_stride_b, p.o_stride_h, p.o_stride_n = out.data_ptr(), out.stride(0), out.stride(1), out.stride(2)
    p.cu_seqlens = ptr(cu)
    keep = []
    if parents is not None:
        par = parents_tensor(parents, dev)
        if par.dim() == 1:
            if par.numel() != N:
                raise RuntimeError(f"parents has {par.numel()} entries for {N} tree nodes")
            p.parents_stride_b = 0
        elif par.dim() == 2 and par.shape == (B, N):
            p.parents_stride_b = par.stride(0)
        else:
            raise RuntimeError(f"parents must be [N] or [B, N], got {tuple(par.shape)}")
        p.mask_kind = _abi.MASK_PARENTS
        p.parents = par.data_ptr()
        p.max_depth = -1 if max_depth is None else int(max_depth)
        keep.append(par)
    else:
        m = tree_mask
        if m.dtype not in (torch.bool, torch.uint8):
            m = m != 0
        if m.dim() == 2:
            m = m.unsqueeze(0)
            msb = 0
        elif m.dim() == 3 and m.shape[0] == B:
            msb = None
        else:
            raise RuntimeError(f"mask must be [N, cols] or [B, N, cols], got {tuple(tree_mask.shape)}")
        m = m.contiguous()
        if msb is None:
            msb = m.stride(0)
        cols = m.shape[2]
        if m.shape[1] != N:
            raise RuntimeError(f"mask has {m.shape[1]} rows for {N} queries")
        # with no prefix (L == N) the two forms mean the same; the tree form
        # is the one the tensor-core kernel takes
        if cols == N:
            p.mask_kind = _abi.MASK_DENSE_TREE
        elif cols == L:
            p.mask_kind = _abi.MASK_DENSE
        else:
            raise RuntimeError(f"mask must have {L} (all kv rows) or {N} (tree rows) columns, got {cols}")
        p.mask = m.data_ptr()
        p.mask_stride_b, p.mask_stride_n = msb, m.stride(1)
        p.max_depth = -1
        keep.append(m)
    p.scale = float(scale) if scale is not None else (1.0 / math.sqrt(D) if D > 0 else 1.0)
    p.lse = ptr(lse)
    p.backend = _BACKENDS[backend]
    p.num_splits = int(num_splits)
    p.kv_rows = kk.shape[0] if cu is not None else 0
    keep += [q4, kk, vv, cu]
    return _Prepared(p, out, lse, keep)
