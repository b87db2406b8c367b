"""ds_moe_decode_noalloc (static device scratch, no workspace) against ds_moe_decode.

Both entry points are called through the C ABI on the same inputs; the
no-allocation variant is called twice in a row (the second call reuses the
static scratch the first one wrote) and each result must match the
workspace entry point within the decode tolerance (relative L2 <= 1e-3).
This file is named so that it is collected last: the scratch array must give
the same answers after every other test has run its kernels.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from deepseeker import _abi, moe, synthetic
from deepseeker._dev import ptr, stream_handle
from oracle import moe as omoe

TOL = 1e-3


def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.double().cpu()
    b = b.double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def noalloc(x: torch.Tensor, layer: moe.MoEWeights, ids: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    out = torch.empty_like(x)
    d = layer.desc(ids.shape[1])
    xdt = _abi.DS_F32 if x.dtype == torch.float32 else _abi.DS_BF16
    _abi.call("ds_moe_decode_noalloc", ctypes.byref(d), ptr(x), xdt, x.shape[0], ptr(ids), ptr(w), ptr(out),
              stream_handle(x.device))
    return out


def routing(T, E, k, seed, device):
    g = torch.Generator().manual_seed(seed)
    w, idx = omoe.route_softmax_topk(torch.randn(T, E, generator=g), k)
    return idx.to(torch.int32).to(device), w.float().to(device)


CASES = [
    # (fmt, H, I, E, k, T, shared_inter, x dtype, scale atoms): FP4 layers
    # with scale atoms reach the tcgen05 kernels (1 and 3 tokens), the FP4
    # layer without atoms at one token the single-token FP4 kernels, q3 its
    # dp2a kernels, f32 x the generic kernels.
    ("fp4", 4096, 2048, 16, 8, 1, 1024, torch.bfloat16, True),
    ("fp4", 2048, 1024, 16, 4, 3, 1024, torch.bfloat16, True),
    ("fp4", 4096, 2048, 16, 8, 1, 1024, torch.bfloat16, False),
    ("q3", 512, 256, 16, 4, 4, 128, torch.bfloat16, False),
    ("fp4", 256, 128, 8, 2, 8, None, torch.float32, False),
]


def status(device) -> int:
    """The no-allocation scratch's error word, read through the C ABI."""
    err = torch.full((1,), -1, dtype=torch.int32).pin_memory()
    _abi.call("ds_moe_decode_noalloc_status", ptr(err), stream_handle(device))
    torch.cuda.synchronize(device)
    return int(err.item())


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c[0]}-H{c[1]}-T{c[5]}-{'atoms' if c[8] else 'plain'}")
def test_noalloc_matches_workspace_entry_point(case, cuda):
    fmt, H, I, E, k, T, Is, dt, atoms = case
    layer = synthetic.make_layer(fmt, H, I, E, seed=41, shared_inter=Is, device=cuda)
    if atoms:
        layer.prepare_tc()
    # the scratch fits every path of these layers: same kernels, same bits
    same_kernels = layer.decode_workspace_bytes(T, k) <= _abi.lib().ds_moe_decode_noalloc_max_scratch()
    torch.manual_seed(7)
    for call in range(2):  # two calls in a row on the shared static scratch
        x = (torch.randn(T, H, device=cuda) * (1.0 + call)).to(dt)
        ids, w = routing(T, E, k, 100 + call, cuda)
        ref = moe.moe_decode(x, layer, ids, w)
        got = noalloc(x, layer, ids, w)
        torch.cuda.synchronize()
        assert torch.isfinite(got.float()).all()
        err = rel_l2(got.float(), ref.float())
        assert err <= TOL, (call, err)
        if same_kernels:
            assert torch.equal(got, ref), call
        assert status(cuda) == 0


@pytest.mark.gpu
def test_noalloc_warm_calls_allocate_nothing(cuda):
    layer = synthetic.make_layer("fp4", 2048, 1024, 16, seed=5, shared_inter=1024, device=cuda).prepare_tc()
    x = torch.randn(1, 2048, device=cuda).to(torch.bfloat16)
    ids, w = routing(1, 16, 4, 3, cuda)
    out = torch.empty_like(x)
    d = layer.desc(4)

    def call():
        _abi.call("ds_moe_decode_noalloc", ctypes.byref(d), ptr(x), _abi.DS_BF16, 1, ptr(ids), ptr(w), ptr(out),
                  stream_handle(cuda))

    call()                                   # first call on the device: symbol-address set-up
    torch.cuda.synchronize()
    torch_before = torch.cuda.memory_allocated(cuda)
    free_before, _ = torch.cuda.mem_get_info(cuda)
    for _ in range(5):
        call()
    torch.cuda.synchronize()
    assert torch.cuda.memory_allocated(cuda) == torch_before
    free_after, _ = torch.cuda.mem_get_info(cuda)
    assert free_after == free_before
    assert status(cuda) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("atoms", [True, False])
def test_noalloc_status_reports_out_of_range_expert(atoms, cuda):
    layer = synthetic.make_layer("fp4", 1024, 1024, 8, seed=2, shared_inter=None, device=cuda)
    if atoms:
        layer.prepare_tc()
    x = torch.randn(1, 1024, device=cuda).to(torch.bfloat16)
    ids = torch.tensor([[1, 8, 3, 2]], dtype=torch.int32, device=cuda)   # 8 is outside [0, 8)
    w = torch.full((1, 4), 0.25, device=cuda)
    got = noalloc(x, layer, ids, w)
    torch.cuda.synchronize()
    assert status(cuda) & 1
    # the bad slot is skipped: the others still produce the layer's output
    ref = moe.moe_decode(x, layer, torch.tensor([[1, -1, 3, 2]], dtype=torch.int32, device=cuda), w)
    assert rel_l2(got.float(), ref.float()) <= TOL
    # the next call clears the word
    noalloc(x, layer, torch.tensor([[1, 0, 3, 2]], dtype=torch.int32, device=cuda), w)
    assert status(cuda) == 0


@pytest.mark.gpu
def test_noalloc_rejects_layers_beyond_the_static_limit(cuda):
    # 8 tokens x top-8 over 64 experts with inter 8192 needs ~17 MB of scratch
    layer = synthetic.make_layer("fp4", 256, 8192, 64, seed=3, device=cuda)
    x = torch.zeros(8, 256, device=cuda, dtype=torch.bfloat16)
    ids = torch.arange(64, device=cuda, dtype=torch.int32).view(8, 8)
    w = torch.full((8, 8), 0.125, device=cuda)
    limit = _abi.lib().ds_moe_decode_noalloc_max_scratch()
    assert limit == 8 << 20
    d = layer.desc(8)
    st = _abi.lib().ds_moe_decode_noalloc(ctypes.byref(d), ptr(x), _abi.DS_BF16, 8, ptr(ids), ptr(w), ptr(x),
                                          stream_handle(cuda))
    assert st == _abi.DS_ERANGE
    assert b"static limit" in _abi.lib().ds_last_error_string()
