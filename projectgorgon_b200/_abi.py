"""ctypes binding of ``libgorgon_b200.so`` (declared in ``include/gorgon_b200.h``).

The library is built in-tree (``projectgorgon_b200/lib``).  Loading fails
loudly when it is missing: there is no CPU or Python fallback for any
operator.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import (POINTER, Structure, c_char_p, c_float, c_int, c_int32, c_int64,
                    c_size_t, c_uint32, c_void_p)
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libgorgon_b200.so"

GORGON_OK = 0
GORGON_ERR_INVALID = 1
GORGON_ERR_UNSUPPORTED = 2
GORGON_ERR_CUDA = 3
GORGON_ERR_WORKSPACE = 4

F32, BF16, F16 = 0, 1, 2
MASK_PARENTS, MASK_DENSE, MASK_DENSE_TREE = 0, 1, 2
BACKEND_AUTO, BACKEND_SIMT, BACKEND_TCGEN05, BACKEND_TCGEN05_PAIR, BACKEND_TCGEN05_CTA = 0, 1, 2, 3, 4

ERR_BAD_PARENT = 1 << 0
ERR_BAD_TRIM_INDEX = 1 << 1
ERR_BAD_VERIFY_INPUT = 1 << 2
ERR_BAD_SEQLEN = 1 << 3
ERR_TIMEOUT = 1 << 4
ERR_CAND_CAPACITY = 1 << 5


class TreeAttnParams(Structure):
    _fields_ = [
        ("dtype", c_int32), ("out_dtype", c_int32),
        ("batch", c_int64), ("heads_q", c_int64), ("heads_kv", c_int64),
        ("n_tree", c_int64), ("kv_len", c_int64), ("head_dim", c_int64),
        ("q", c_void_p), ("q_stride_b", c_int64), ("q_stride_h", c_int64), ("q_stride_n", c_int64),
        ("k", c_void_p), ("k_stride_b", c_int64), ("k_stride_h", c_int64), ("k_stride_s", c_int64),
        ("v", c_void_p), ("v_stride_b", c_int64), ("v_stride_h", c_int64), ("v_stride_s", c_int64),
        ("out", c_void_p), ("o_stride_b", c_int64), ("o_stride_h", c_int64), ("o_stride_n", c_int64),
        ("cu_seqlens", c_void_p),
        ("mask_kind", c_int32),
        ("parents", c_void_p), ("parents_stride_b", c_int64),
        ("max_depth", c_int32),
        ("mask", c_void_p), ("mask_stride_b", c_int64), ("mask_stride_n", c_int64),
        ("scale", c_float),
        ("lse", c_void_p),
        ("backend", c_int32),
        ("num_splits", c_int32),
        ("kv_rows", c_int64),
    ]


class VerifyParams(Structure):
    _fields_ = [
        ("dtype", c_int32),
        ("logits", c_void_p), ("logits_stride_b", c_int64), ("logits_stride_r", c_int64),
        ("batch", c_int64), ("rows", c_int64), ("vocab", c_int64), ("n", c_int64),
        ("prompt_len", c_int64),
        ("draft", c_void_p), ("draft_stride_b", c_int64),
        ("parents", c_void_p), ("parents_stride_b", c_int64),
        ("pred", c_void_p), ("accepted_len", c_void_p), ("path", c_void_p),
        ("bonus", c_void_p), ("best_node", c_void_p), ("hidden_row", c_void_p),
    ]


class KvTrimParams(Structure):
    _fields_ = [
        ("elem_bytes", c_int32),
        ("layers", c_int64), ("batch", c_int64), ("heads", c_int64),
        ("seq_capacity", c_int64), ("head_dim", c_int64),
        ("stride_b", c_int64), ("stride_h", c_int64), ("stride_s", c_int64),
        ("k_src", POINTER(c_void_p)), ("v_src", POINTER(c_void_p)),
        ("k_dst", POINTER(c_void_p)), ("v_dst", POINTER(c_void_p)),
        ("src_idx", c_void_p), ("idx_stride_b", c_int64), ("max_len", c_int64),
        ("lens", c_void_p),
        ("dst_start", c_void_p),
    ]


class CandidateTreeParams(Structure):
    _fields_ = [
        ("dtype", c_int32),
        ("logits", c_void_p), ("logits_stride_b", c_int64), ("logits_stride_l", c_int64),
        ("batch", c_int64), ("levels", c_int64), ("vocab", c_int64),
        ("top_k", c_int32),
        ("max_candidates", c_int32),
        ("confidence_threshold", c_float),
        ("use_path_confidence", c_int32), ("entropy_weighted", c_int32),
        ("max_nodes", c_int64),
        ("tokens", c_void_p), ("parents", c_void_p), ("probs", c_void_p), ("n_nodes", c_void_p),
        ("topk_ids", c_void_p), ("topk_scores", c_void_p), ("topk_probs", c_void_p), ("entropy", c_void_p),
    ]


class HeadCandidateParams(Structure):
    _fields_ = [
        ("tree", CandidateTreeParams),
        ("x_dtype", c_int32),
        ("hidden", c_void_p), ("hidden_stride_b", c_int64), ("hidden_stride_l", c_int64),
        ("hidden_size", c_int64),
        ("lm_head", c_void_p), ("lm_head_stride_v", c_int64),
    ]


MAX_PEERS = 8  # GORGON_MAX_PEERS


class IpcHandle(Structure):
    _fields_ = [("bytes", ctypes.c_ubyte * 64)]


class PeerGroup(Structure):
    _fields_ = [("world", c_int32), ("rank", c_int32), ("base", c_void_p * MAX_PEERS),
                ("signal_offset", c_int64)]


# Every symbol the header declares, with its ctypes signature.
SIGNATURES = {
    "gorgon_abi_version": (c_int, []),
    "gorgon_last_error": (c_char_p, []),
    "gorgon_device_error": (c_int, [POINTER(c_uint32), c_int]),
    "gorgon_set_wait_limit_ns": (c_int64, [c_int64]),
    "gorgon_tree_mask": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_int64, c_void_p, c_void_p]),
    "gorgon_tree_attn_workspace_size": (c_size_t, [POINTER(TreeAttnParams)]),
    "gorgon_tree_attn": (c_int, [POINTER(TreeAttnParams), c_void_p, c_size_t, c_void_p]),
    "gorgon_tree_attn_plan": (c_int, [POINTER(TreeAttnParams), POINTER(c_int32), POINTER(c_int32),
                                      POINTER(c_int32)]),
    "gorgon_peer_buffer_alloc": (c_int, [c_size_t, POINTER(c_void_p), POINTER(IpcHandle)]),
    "gorgon_peer_buffer_open": (c_int, [POINTER(IpcHandle), POINTER(c_void_p)]),
    "gorgon_peer_buffer_close": (c_int, [c_void_p]),
    "gorgon_peer_buffer_free": (c_int, [c_void_p]),
    "gorgon_tree_attn_gather": (c_int, [POINTER(TreeAttnParams), POINTER(PeerGroup), c_void_p, c_size_t,
                                        c_void_p]),
    "gorgon_verify_workspace_size": (c_size_t, [POINTER(VerifyParams)]),
    "gorgon_verify": (c_int, [POINTER(VerifyParams), c_void_p, c_size_t, c_void_p]),
    "gorgon_verify_noalloc": (c_int, [POINTER(VerifyParams), c_void_p]),
    "gorgon_kv_trim": (c_int, [POINTER(KvTrimParams), c_void_p]),
    "gorgon_candidate_tree_workspace_size": (c_size_t, [POINTER(CandidateTreeParams)]),
    "gorgon_candidate_tree": (c_int, [POINTER(CandidateTreeParams), c_void_p, c_size_t, c_void_p]),
    "gorgon_head_candidate_tree_workspace_size": (c_size_t, [POINTER(HeadCandidateParams)]),
    "gorgon_head_candidate_tree": (c_int, [POINTER(HeadCandidateParams), c_void_p, c_size_t, c_void_p]),
}

_lib = None


class GorgonError(RuntimeError):
    """A call into the CUDA library failed (RuntimeError, as TORCH_CHECK raises)."""


def lib() -> ctypes.CDLL:
    """The loaded library; raises if it has not been built."""
    global _lib
    if _lib is None:
        path = Path(os.environ.get("GORGON_B200_LIB", LIB_PATH))
        if not path.exists():
            raise ImportError(
                f"{path} is missing: build the CUDA library first "
                "(python -m projectgorgon_b200._build or __graft_entry__.build())")
        handle = ctypes.CDLL(str(path))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(rc: int, what: str) -> None:
    if rc == GORGON_OK:
        return
    msg = lib().gorgon_last_error().decode(errors="replace")
    raise GorgonError(f"{what} failed ({rc}): {msg}")


def device_error(clear: bool = True) -> int:
    """Synchronously reads (and by default clears) the device error word."""
    flags = c_uint32(0)
    check(lib().gorgon_device_error(ctypes.byref(flags), int(clear)), "gorgon_device_error")
    return int(flags.value)


def set_wait_limit_ns(ns: int) -> int:
    """Sets the bound on every wait inside the tensor-core kernels (process
    wide, nanoseconds; <= 0 leaves it unchanged) and returns the previous one."""
    return int(lib().gorgon_set_wait_limit_ns(int(ns)))


def pointer_array(ptrs) -> ctypes.Array:
    arr = (c_void_p * len(ptrs))()
    for i, p in enumerate(ptrs):
        arr[i] = p
    return arr
