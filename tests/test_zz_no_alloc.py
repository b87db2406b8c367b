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
    # (fmt, H, I, E, k, T, shared_inter, x dtype): the first reaches the
    # single-token tensor-core kernels, the others the generic kernels.
    ("fp4", 4096, 2048, 16, 8, 1, 1024, torch.bfloat16),
    ("q3", 512, 256, 16, 4, 4, 128, torch.bfloat16),
    ("fp4", 256, 128, 8, 2, 8, None, torch.float32),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c[0]}-H{c[1]}-T{c[5]}")
def test_noalloc_matches_workspace_entry_point(case, cuda):
    fmt, H, I, E, k, T, Is, dt = case
    layer = synthetic.make_layer(fmt, H, I, E, seed=41, shared_inter=Is, device=cuda)
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
