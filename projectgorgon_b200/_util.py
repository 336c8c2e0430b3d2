"""Small torch-side helpers shared by the operator modules."""
from __future__ import annotations

from typing import Iterable, List, Sequence, Union

import torch

from . import _abi

_DT = {torch.float32: _abi.F32, torch.bfloat16: _abi.BF16, torch.float16: _abi.F16}


def gorgon_dtype(dt: torch.dtype) -> int:
    try:
        return _DT[dt]
    except KeyError:
        raise RuntimeError(f"unsupported dtype {dt}: expected float32, bfloat16 or float16") from None


def require_cuda(what: str, *tensors: torch.Tensor) -> None:
    """ValueError for host tensors, as the reference wrappers raise
    (src/gorgon/kernels/tree_attention_triton.py:92-93)."""
    for t in tensors:
        if not (isinstance(t, torch.Tensor) and t.is_cuda):
            raise ValueError(f"{what} must be CUDA tensors.")


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_ptr(device: torch.device) -> int:
    """The cudaStream_t of torch's current stream on `device`, as an int
    (the raw accessor skips building a Stream object on every call)."""
    if _raw_stream is not None and device.index is not None:
        return _raw_stream(device.index)
    return torch.cuda.current_stream(device).cuda_stream


class _NoSwitch:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


_NO_SWITCH = _NoSwitch()


def on_device(device: torch.device):
    """`torch.cuda.device(device)`, or nothing when it is already current."""
    if device.index is None or torch.cuda.current_device() == device.index:
        return _NO_SWITCH
    return torch.cuda.device(device)


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    """Caller-owned scratch from torch's caching allocator (stream-ordered)."""
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


def parents_tensor(parents: Union[Sequence[int], torch.Tensor], device: torch.device) -> torch.Tensor:
    """int32 device copy of a parents list or tensor
    (src/gorgon/kernels/fused_tree_verify_triton.py:140-143)."""
    if isinstance(parents, torch.Tensor):
        return parents.to(device=device, dtype=torch.int32).contiguous()
    return torch.tensor(list(parents), dtype=torch.int32, device=device)


def ptr(t: torch.Tensor) -> int:
    return t.data_ptr() if t is not None else 0
