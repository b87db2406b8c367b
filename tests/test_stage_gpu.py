"""ds_copy_ranges / ds_host_device_pointer: the kernel that stages a
host-fed decode step's inputs and output through pinned host memory."""
from __future__ import annotations

import ctypes

import pytest
import torch

from deepseeker import _abi, moe

pytestmark = pytest.mark.gpu


def test_round_trip_through_pinned_memory(cuda):
    g = torch.Generator().manual_seed(3)
    sizes = [8192, 1024, 16, 48 * 1024]                      # bytes, multiples of 16
    src = [torch.randint(0, 256, (n,), dtype=torch.uint8, generator=g).pin_memory() for n in sizes]
    mid = [torch.zeros(n, dtype=torch.uint8, device="cuda") for n in sizes]
    back = [torch.zeros(n, dtype=torch.uint8).pin_memory() for n in sizes]
    moe.copy_ranges([(m.data_ptr(), moe.host_device_pointer(s), s.numel()) for m, s in zip(mid, src)], "cuda")
    moe.copy_ranges([(moe.host_device_pointer(b), m.data_ptr(), m.numel()) for b, m in zip(back, mid)], "cuda")
    moe.wait_stream("cuda")
    for s, m, b in zip(src, mid, back):
        assert torch.equal(m.cpu(), s)
        assert torch.equal(b, s)


def test_rejects_unmapped_and_misaligned(cuda):
    plain = torch.zeros(64, dtype=torch.uint8)               # pageable: no device mapping
    d = ctypes.c_void_p(0)
    with pytest.raises(ValueError):
        _abi.call("ds_host_device_pointer", ctypes.c_void_p(plain.data_ptr()), ctypes.byref(d))
    a = torch.zeros(64, dtype=torch.uint8, device="cuda")
    b = torch.zeros(64, dtype=torch.uint8, device="cuda")
    with pytest.raises(ValueError):
        moe.copy_ranges([(a.data_ptr() + 8, b.data_ptr(), 32)], "cuda")
    with pytest.raises(ValueError):
        moe.copy_ranges([(a.data_ptr(), b.data_ptr(), 24)], "cuda")
