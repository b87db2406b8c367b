"""Sort-and-pad alignment of routed (token, slot) pairs, on the GPU.

Drop-in for ``deepseeker.moe_align`` (src/deepseeker/moe_align.py:21-46):
same contract, same return types (int64 numpy arrays and an int), same
ValueErrors; the work runs in ``ds_moe_align`` (moe_align.cu).
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _abi
from ._dev import ptr, stream_handle

MAX_EXPERTS = 1024


def align_block_size_device(topk_ids: torch.Tensor, block_size: int, num_experts: int
                            ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Device form: topk_ids [M, K] int32 CUDA tensor -> (sorted_ids, expert_ids, n_pad)
    as int32 CUDA tensors sized to capacity; n_pad[0] is the padded length
    (-1 when an id is out of range)."""
    if topk_ids.dim() != 2:
        raise ValueError(f"topk_ids must be 2-D, got shape {tuple(topk_ids.shape)}")
    if block_size < 1 or num_experts < 1:
        raise ValueError("block_size and num_experts must be >= 1")
    if num_experts > MAX_EXPERTS:
        raise NotImplementedError(f"num_experts > {MAX_EXPERTS}")
    ids = topk_ids.to(torch.int32).contiguous()
    m, k = ids.shape
    cap, bcap = ctypes.c_int64(0), ctypes.c_int64(0)
    _abi.call("ds_moe_align_capacity", m, k, num_experts, block_size, ctypes.byref(cap), ctypes.byref(bcap))
    dev = ids.device
    sorted_ids = torch.empty(max(cap.value, 1), dtype=torch.int32, device=dev)
    expert_ids = torch.empty(max(bcap.value, 1), dtype=torch.int32, device=dev)
    n_pad = torch.empty(1, dtype=torch.int32, device=dev)
    _abi.call("ds_moe_align", ptr(ids), m, k, num_experts, block_size, ptr(sorted_ids), cap.value,
              ptr(expert_ids), bcap.value, ptr(n_pad), stream_handle(dev))
    return sorted_ids, expert_ids, n_pad


def align_block_size(topk_ids: np.ndarray, block_size: int, num_experts: int,
                     device: torch.device | str = "cuda") -> tuple[np.ndarray, np.ndarray, int]:
    """Sort flat (token, top-k) positions by expert with block padding."""
    topk_ids = np.asarray(topk_ids)
    if topk_ids.ndim != 2:
        raise ValueError(f"topk_ids must be 2-D, got shape {topk_ids.shape}")
    if block_size < 1 or num_experts < 1:
        raise ValueError("block_size and num_experts must be >= 1")
    flat = topk_ids.reshape(-1)
    if flat.size and (flat.min() < 0 or flat.max() >= num_experts):
        raise ValueError("expert ids out of range")
    if flat.size == 0:
        return np.zeros(0, np.int64), np.zeros(0, np.int64), 0
    ids = torch.from_numpy(np.ascontiguousarray(topk_ids, dtype=np.int32)).to(device)
    s, e, n = align_block_size_device(ids, block_size, num_experts)
    n_pad = int(n.item())
    if n_pad < 0:
        raise ValueError("expert ids out of range")
    return (s[:n_pad].cpu().numpy().astype(np.int64), e[:n_pad // block_size].cpu().numpy().astype(np.int64),
            n_pad)
