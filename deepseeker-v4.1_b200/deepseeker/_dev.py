"""Small helpers for passing torch tensors through the C ABI."""
from __future__ import annotations

import ctypes

import numpy as np
import torch


def stream_handle(device: torch.device | None = None) -> ctypes.c_void_p:
    """cudaStream_t of torch's current stream on `device`."""
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def ptr(t: torch.Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def require_cuda(t: torch.Tensor, name: str, dtype: torch.dtype | tuple | None = None) -> torch.Tensor:
    """Check that `t` is a CUDA tensor of the given dtype; return it contiguous."""
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if dtype is not None:
        allowed = dtype if isinstance(dtype, tuple) else (dtype,)
        if t.dtype not in allowed:
            raise ValueError(f"{name} must have dtype {allowed}, got {t.dtype}")
    return t.contiguous()


def device_of(*ts: torch.Tensor) -> torch.device:
    for t in ts:
        if isinstance(t, torch.Tensor) and t.is_cuda:
            return t.device
    return torch.device("cuda", torch.cuda.current_device())


def to_device(a, device: torch.device | None = None, dtype: torch.dtype | None = None) -> torch.Tensor:
    """numpy array / bytes / tensor -> contiguous CUDA tensor (host data is copied)."""
    if isinstance(a, (bytes, bytearray, memoryview)):
        a = np.frombuffer(a, dtype=np.uint8)
    if isinstance(a, np.ndarray):
        a = np.ascontiguousarray(a)
        if not a.flags.writeable:    # torch wants writable storage; the data is copied to the device anyway
            a = a.copy()
        t = torch.from_numpy(a)
    else:
        t = a
    if dtype is not None and t.dtype != dtype:
        t = t.to(dtype)
    return t.to(device or torch.device("cuda"), non_blocking=False).contiguous()
