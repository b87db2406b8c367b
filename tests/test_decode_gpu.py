"""Fused decode MoE layer (ds_moe_decode) vs the torch fp32 oracle.

Weights are built on the device by the seeded synthetic builder, read back,
dequantised by the oracle and run through ``oracle.moe.moe_combine`` (the
restatement of moe_layer's expert loop, mlx_forward.py:388-419).
Tolerance: relative L2 <= 1e-3; f32-output runs are also
held to 1e-5, which is what fp32 accumulation actually delivers.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from deepseeker import moe, synthetic
from oracle import fp4 as ofp4
from oracle import moe as omoe
from oracle import q3 as oq3

pytestmark = pytest.mark.gpu

TOL = 1e-3


def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.double().cpu()
    b = b.double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def dense_expert(bank: moe.ExpertBank, e: int) -> torch.Tensor:
    if bank.fmt == 0:  # FP4
        return torch.from_numpy(ofp4.dequant_matrix(bank.data[e].cpu().numpy(), bank.scales[e].cpu().numpy()))
    w = bank.data[e].cpu().numpy().view(np.uint32)
    return torch.from_numpy(oq3.dequant(w, bank.scales[e].cpu().numpy(), bank.biases[e].cpu().numpy()))


def oracle_out(x, ids, wts, layer: moe.MoEWeights, limit):
    cache = {}

    def ew(e):
        if e not in cache:
            cache[e] = tuple(dense_expert(b, e) for b in (layer.w1, layer.w3, layer.w2))
        return cache[e]
    shared = None
    if layer.shared_w1 is not None:
        shared = (layer.shared_w1.cpu(), layer.shared_w3.cpu(), layer.shared_w2.cpu())
    return omoe.moe_combine(x.cpu(), ids.cpu().long(), wts.cpu(), ew, shared=shared, limit=limit)


def routing(T, E, k, seed):
    g = torch.Generator().manual_seed(seed)
    w, idx = omoe.route_softmax_topk(torch.randn(T, E, generator=g), k)
    return idx.to(torch.int32), w


@pytest.mark.parametrize("fmt", ["fp4", "q3"])
@pytest.mark.parametrize("T", [1, 3, 8])
def test_small_layer(fmt, T, cuda):
    H, I, E, k = 256, 128, 16, 4
    layer = synthetic.make_layer(fmt, H, I, E, seed=5 + T, shared_inter=192, std=0.05)
    ids, wts = routing(T, E, k, seed=T)
    g = torch.Generator().manual_seed(100 + T)
    x32 = torch.randn(T, H, generator=g)
    x = x32.to(torch.bfloat16)
    out = moe.moe_decode(x.cuda(), layer, ids.cuda(), wts.cuda())
    ref = oracle_out(x, ids, wts, layer, 10.0)
    assert out.dtype == torch.bfloat16 and out.shape == (T, H)
    assert rel_l2(out, ref) < TOL
    # f32 activations / output: the same kernels, no bf16 rounding of the result
    out32 = moe.moe_decode(x32.cuda(), layer, ids.cuda(), wts.cuda())
    ref32 = oracle_out(x32, ids, wts, layer, 10.0)
    assert rel_l2(out32, ref32) < 1e-5


@pytest.mark.parametrize("fmt", ["fp4", "q3"])
def test_shared_experts_dropped_slots_and_no_clamp(fmt, cuda):
    H, I, E, k = 128, 64, 8, 3
    layer = synthetic.make_layer(fmt, H, I, E, seed=21, shared_inter=None, std=0.2, limit=None)
    # token 0 and 1 share expert 5; token 1 has a dropped slot (-1); token 2 repeats an expert
    ids = torch.tensor([[5, 2, 7], [1, -1, 5], [3, 3, 0]], dtype=torch.int32)
    wts = torch.tensor([[0.5, 0.3, 0.2], [0.6, 0.0, 0.4], [0.7, 0.1, 0.2]])
    x32 = torch.randn(3, H, generator=torch.Generator().manual_seed(3)) * 4.0
    out = moe.moe_decode(x32.cuda(), layer, ids.cuda(), wts.cuda())
    ref = oracle_out(x32, ids, wts, layer, None)
    assert rel_l2(out, ref) < 1e-5


def test_gate_after_down_semantics(cuda):
    """grouped_swiglu multiplies the gate after the down projection (grouped.py:50-53)."""
    H, I, E, k = 128, 64, 8, 2
    layer = synthetic.make_layer("fp4", H, I, E, seed=8, shared_inter=None, std=0.1, limit=None)
    layer.route_before_down = False
    ids, wts = routing(2, E, k, seed=9)
    x32 = torch.randn(2, H, generator=torch.Generator().manual_seed(1))
    out = moe.moe_decode(x32.cuda(), layer, ids.cuda(), wts.cuda())
    ref = oracle_out(x32, ids, wts, layer, None)
    assert rel_l2(out, ref) < 1e-5


def test_reference_geometry(cuda):
    """DeepSeek-V4.1-Flash expert shapes: hidden 5120, inter 2304, top-6, sqrt-softplus router."""
    H, I, E, k = 5120, 2304, 12, 6
    layer = synthetic.make_layer("fp4", H, I, E, seed=31, shared_inter=2304, std=0.02)
    g = torch.Generator().manual_seed(4)
    x = torch.randn(1, H, generator=g).to(torch.bfloat16)
    gate_w = torch.randn(E, H, generator=g) * 0.02
    gate_b = torch.randn(E, generator=g) * 0.01
    out = moe.moe_layer(x.cuda(), gate_w.cuda(), gate_b.cuda(), layer.resident(), layer.shared_expert(), top_k=k)
    scores = omoe.sqrtsoftplus_scores(x, gate_w)
    wts, idx = omoe.route_topk(scores, gate_b, k)
    ref = oracle_out(x, idx.to(torch.int32), wts, layer, 10.0)
    assert rel_l2(out, ref) < TOL


def test_config1_single_expert_f32(cuda):
    """1 token, hidden 4096, inter 2048, x ~ N(0,1) f32,
    W ~ N(0, 0.02) -> FP4, out = down(silu(gate x) * up x), seed 0."""
    H, I = 4096, 2048
    layer = synthetic.make_layer("fp4", H, I, 1, seed=0, shared_inter=None, std=0.02, limit=None)
    x = torch.randn(1, H, generator=torch.Generator().manual_seed(0))
    ids = torch.zeros(1, 1, dtype=torch.int32)
    wts = torch.ones(1, 1)
    out = moe.moe_decode(x.cuda(), layer, ids.cuda(), wts.cuda())
    w1, w3, w2 = (dense_expert(b, 0) for b in (layer.w1, layer.w3, layer.w2))
    ref = omoe.expert_ffn(x, w1, w3, w2, limit=None)
    assert rel_l2(out, ref) < 1e-5


@pytest.mark.parametrize("fmt,T", [("fp4", 1), ("q3", 1), ("q3", 4), ("q3", 8)])
def test_config2_3_full_layer(fmt, T, cuda):
    """BASELINE configs 2/3: hidden 4096, 256 experts (inter 2048), top-8 softmax,
    bf16 shared expert, bf16 activations; all experts resident."""
    H, I, E, k = 4096, 2048, 256, 8
    layer = synthetic.make_layer(fmt, H, I, E, seed=2, shared_inter=2048, std=0.02)
    ids, wts = routing(T, E, k, seed=12)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(13)).to(torch.bfloat16)
    out = moe.moe_decode(x.cuda(), layer, ids.cuda(), wts.cuda())
    ref = oracle_out(x, ids, wts, layer, 10.0)
    assert rel_l2(out, ref) < TOL
    # reruns are bitwise identical (deterministic combine)
    again = moe.moe_decode(x.cuda(), layer, ids.cuda(), wts.cuda())
    assert torch.equal(out, again)


def test_invalid_arguments(cuda):
    layer = synthetic.make_layer("fp4", 128, 64, 4, seed=1, shared_inter=None)
    x = torch.zeros(9, 128, dtype=torch.bfloat16, device="cuda")
    ids = torch.zeros(9, 2, dtype=torch.int32, device="cuda")
    with pytest.raises(ValueError):
        moe.moe_decode(x, layer, ids, torch.ones(9, 2, device="cuda"))
    with pytest.raises(ValueError):
        moe.moe_decode(x[:1, :64].contiguous(), layer, ids[:1], torch.ones(1, 2, device="cuda"))


# ---------------------------------------------------------------- single token, FP4 banks without scale atoms

@pytest.mark.parametrize("k,shared", [(4, True), (3, True), (5, False), (1, True)])
def test_single_token_path(k, shared, cuda):
    """One bf16 token over FP4 banks without scale atoms runs on the
    register-dequant kernel; odd slot counts, no shared expert and top-1
    exercise its task bookkeeping."""
    H, I, E = 1024, 512, 16
    layer = synthetic.make_layer("fp4", H, I, E, seed=40 + k, shared_inter=1024 if shared else None, std=0.05)
    for seed in range(3):
        ids, wts = routing(1, E, k, seed=seed)
        x = torch.randn(1, H, generator=torch.Generator().manual_seed(seed)).to(torch.bfloat16)
        out = moe.moe_decode(x.cuda(), layer, ids.cuda(), wts.cuda())
        ref = oracle_out(x, ids, wts, layer, 10.0)
        assert rel_l2(out, ref) < TOL, (seed, rel_l2(out, ref))


def test_single_token_dropped_and_duplicate_slots(cuda):
    H, I, E = 2048, 1024, 8
    layer = synthetic.make_layer("fp4", H, I, E, seed=77, shared_inter=1024, std=0.05)
    ids = torch.tensor([[6, -1, 2, 6]], dtype=torch.int32)     # dropped slot, duplicate expert
    wts = torch.tensor([[0.5, 0.2, 0.3, 0.9]])
    x = torch.randn(1, H, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
    out = moe.moe_decode(x.cuda(), layer, ids.cuda(), wts.cuda())
    ref = oracle_out(x, ids, wts, layer, 10.0)
    assert rel_l2(out, ref) < TOL
    ids = torch.full((1, 4), -1, dtype=torch.int32)             # nothing routed: shared expert only
    out = moe.moe_decode(x.cuda(), layer, ids.cuda(), wts.cuda())
    ref = oracle_out(x, ids, wts, layer, 10.0)
    assert rel_l2(out, ref) < TOL


def test_single_token_matches_generic_path(cuda):
    """Token 0 through the single-token FP4 kernels (one-token call) and through
    the generic kernels (the same token as row 0 of a two-token call, FP4
    banks without scale atoms) agrees to well inside the tolerance."""
    layer = synthetic.make_layer("fp4", 1024, 512, 16, seed=3, shared_inter=1024, std=0.05)
    w, ids = omoe.route_softmax_topk(torch.randn(2, 16, generator=torch.Generator().manual_seed(1)), 4)
    x = torch.randn(2, 1024, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16).cuda()
    ids, w = ids.to(torch.int32).cuda(), w.cuda()
    one = moe.moe_decode(x[:1].contiguous(), layer, ids[:1].contiguous(), w[:1].contiguous())
    two = moe.moe_decode(x, layer, ids, w)
    assert rel_l2(one[0], two[0]) < 2e-3


def test_single_token_no_routes_no_shared_is_zero(cuda):
    layer = synthetic.make_layer("fp4", 1024, 512, 8, seed=9, shared_inter=None, std=0.05)
    ids = torch.full((1, 2), -1, dtype=torch.int32, device="cuda")
    out = torch.full((1, 1024), 7.0, dtype=torch.bfloat16, device="cuda")
    moe.moe_decode(torch.ones(1, 1024, dtype=torch.bfloat16, device="cuda"), layer, ids,
                   torch.ones(1, 2, device="cuda"), out=out)
    assert bool((out == 0).all())
