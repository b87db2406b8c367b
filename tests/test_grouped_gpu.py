"""Grouped expert FFN on the GPU.

* Dense drop-in (grouped_swiglu / naive_swiglu, ds_dense_swiglu) against the
  reference test's cases (tests/test_grouped.py:16-58) and the CPU oracle.
* FP4 and q3 banks through the tcgen05 path (ds_grouped_ffn) against a
  float64 torch reference built from the bit-exact device dequant, output
  rounded to bf16 like the reference layer (mlx_forward.py:388-419 semantics
  with the clamp and the route weight before the down projection;
  grouped.py:34-56 semantics without clamp and with the weight after it);
  small q3 cases also against the CPU oracle (oracle.moe.moe_combine on
  oracle.q3's dequant).  Tolerance: relative L2 <= 1e-3.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from deepseeker import grouped, metal_fp4, mlx_weights, moe, synthetic
from oracle import moe as omoe
from oracle import q3 as oq3

pytestmark = pytest.mark.gpu

TOL = 1e-3


def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.double().cpu()
    b = b.double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


# ---------------------------------------------------------------- dense drop-in

def tiny_weights(device):
    g = torch.Generator().manual_seed(0)
    weights = {}
    for expert in range(4):
        gate = torch.randn(16, 8, generator=g) * 0.1
        up = torch.randn(16, 8, generator=g) * 0.1
        down = torch.randn(8, 16, generator=g) * 0.1
        weights[expert] = (gate.to(device), up.to(device), down.to(device))
    x = torch.randn(5, 16, generator=g).to(device)
    return weights, x


def test_dense_grouped_matches_naive_and_oracle(cuda):
    weights, x = tiny_weights(cuda)
    topk = [[3, 1], [0, 2], [1, 1], [2, 3], [0, 3]]
    router = [[0.6, 0.4]] * 5
    groups = grouped.plan_groups(topk, 4)
    ref = grouped.naive_swiglu(x, weights, topk, router)
    got = grouped.grouped_swiglu(x, weights, groups, router)
    assert float((ref - got).abs().max()) < 1e-4
    cpu_w = {e: tuple(t.cpu() for t in w) for e, w in weights.items()}
    ora = omoe.grouped_swiglu(x.cpu(), cpu_w, omoe.plan_groups(topk, 4), router)
    assert float((got.cpu() - ora).abs().max()) < 1e-5
    ora_n = omoe.naive_swiglu(x.cpu(), cpu_w, topk, router)
    assert float((ref.cpu() - ora_n).abs().max()) < 1e-5


def test_dense_grouped_without_router(cuda):
    weights, x = tiny_weights(cuda)
    topk = [[0, 1], [2, 3]]
    groups = grouped.plan_groups(topk, 4)
    ref = grouped.naive_swiglu(x[:2], weights, topk)
    got = grouped.grouped_swiglu(x[:2], weights, groups)
    assert float((ref - got).abs().max()) < 1e-4


# ---------------------------------------------------------------- FP4 banks, tcgen05 path

def dense(bank: moe.ExpertBank, e: int) -> torch.Tensor:
    """Expert e of a bank as f64 [rows, cols], from the bit-exact device dequant."""
    if bank.fmt == 0:
        return metal_fp4.dequant(bank.data[e], bank.scales[e]).view(bank.rows, bank.cols).double()
    return mlx_weights.dequant_q3(bank.data[e], bank.scales[e], bank.biases[e]).double()


def torch_reference(x, layer: moe.MoEWeights, ids, w, limit, before):
    """float64 reference; weights from the bit-exact device dequant."""
    T, H = x.shape
    xd = x.double()
    out = torch.zeros(T, H, dtype=torch.float64, device=x.device)
    for e in torch.unique(ids[ids >= 0]).tolist():
        rows, slots = torch.nonzero(ids == e, as_tuple=True)
        w1, w3, w2 = dense(layer.w1, e), dense(layer.w3, e), dense(layer.w2, e)
        xr = xd[rows]
        g = xr @ w1.T
        u = xr @ w3.T
        if limit:
            g = g.clamp(max=limit)
            u = u.clamp(-limit, limit)
        h = g / (1 + torch.exp(-g)) * u
        gw = w[rows, slots].double()[:, None]
        if before:
            h = h * gw
        y = h @ w2.T
        if not before:
            y = y * gw
        out.index_add_(0, rows, y)
    return out.to(torch.bfloat16)


def run_case(cuda, H, I, E, k, T, limit, before, seed, zipf=False, drop=0.0, fmt="fp4"):
    layer = synthetic.make_layer(fmt, H, I, E, seed=seed, shared_inter=None, device=cuda, limit=limit)
    g = torch.Generator(device=cuda).manual_seed(seed)
    x = torch.randn(T, H, generator=g, device=cuda).to(torch.bfloat16)
    if zipf:
        ids, w = synthetic.zipf_routing(T, E, k, seed=seed, device=cuda)
    else:
        w, ids = omoe.route_softmax_topk(torch.randn(T, E, generator=g, device=cuda), k)
        ids = ids.to(torch.int32)
    if drop:
        mask = torch.rand(T, k, generator=g, device=cuda) < drop
        ids = torch.where(mask, torch.full_like(ids, -1), ids)
    ffn = grouped.GroupedFFN(layer, k)
    got = ffn(x, ids, w.float(), route_before_down=before)
    ref = torch_reference(x, layer, ids, w.float(), limit, before)
    return got, ref, ffn, x, ids, w


@pytest.mark.parametrize("before,limit", [(True, 10.0), (False, None)])
def test_fp4_small(before, limit, cuda):
    got, ref, *_ = run_case(cuda, 256, 256, 8, 2, 37, limit, before, seed=11)
    assert torch.isfinite(got.float()).all()
    assert rel_l2(got, ref) <= TOL


def test_fp4_medium_zipf_with_dropped_slots(cuda):
    got, ref, *_ = run_case(cuda, 1024, 512, 32, 4, 300, 10.0, True, seed=12, zipf=True, drop=0.1)
    assert rel_l2(got, ref) <= TOL


def test_fp4_config4_full(cuda):
    """2048 tokens, hidden 4096, 256 experts (inter 2048), top-8 Zipf(1.1)."""
    got, ref, ffn, x, ids, w = run_case(cuda, 4096, 2048, 256, 8, 2048, 10.0, True, seed=4, zipf=True)
    assert rel_l2(got, ref) <= TOL
    again = ffn(x, ids, w.float(), route_before_down=True)
    assert torch.equal(again, got), "grouped path must be deterministic"


def test_fp4_matches_decode_path(cuda):
    """Same layer through the decode kernels (validated against the CPU oracle)."""
    layer = synthetic.make_layer("fp4", 4096, 2048, 64, seed=21, shared_inter=None, device=cuda)
    g = torch.Generator(device=cuda).manual_seed(21)
    x = torch.randn(8, 4096, generator=g, device=cuda).to(torch.bfloat16)
    w, ids = omoe.route_softmax_topk(torch.randn(8, 64, generator=g, device=cuda), 8)
    ids = ids.to(torch.int32)
    got = grouped.GroupedFFN(layer, 8)(x, ids, w.float(), route_before_down=True)
    dec = moe.moe_decode(x, layer, ids, w.float())
    assert rel_l2(got, dec) <= TOL


def test_fp4_out_of_range_expert_gives_nan_not_fault(cuda):
    layer = synthetic.make_layer("fp4", 256, 256, 8, seed=5, shared_inter=None, device=cuda)
    x = torch.randn(4, 256, device=cuda).to(torch.bfloat16)
    ids = torch.tensor([[0, 1], [2, 9], [3, 4], [5, 6]], dtype=torch.int32, device=cuda)
    w = torch.full((4, 2), 0.5, device=cuda)
    out = grouped.GroupedFFN(layer, 2)(x, ids, w)
    torch.cuda.synchronize()
    assert torch.isnan(out.float()).all()


# ---------------------------------------------------------------- q3 banks, tcgen05 path (codes exact in e4m3)

@pytest.mark.parametrize("before,limit", [(True, 10.0), (False, None)])
def test_q3_small(before, limit, cuda):
    got, ref, *_ = run_case(cuda, 256, 256, 8, 2, 37, limit, before, seed=11, fmt="q3")
    assert torch.isfinite(got.float()).all()
    assert rel_l2(got, ref) <= TOL


def test_q3_small_vs_cpu_oracle(cuda):
    """The same layer through the CPU oracle: oracle.q3 dequant of the bank
    words, oracle.moe.moe_combine (mlx_forward.py:388-419)."""
    H, I, E, k, T = 256, 384, 8, 3, 21
    layer = synthetic.make_layer("q3", H, I, E, seed=5, shared_inter=None, device=cuda, limit=10.0)
    g = torch.Generator().manual_seed(6)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    w, ids = omoe.route_softmax_topk(torch.randn(T, E, generator=g), k)
    ids = ids.to(torch.int32)
    got = grouped.GroupedFFN(layer, k)(x.to(cuda), ids.to(cuda), w.float().to(cuda), route_before_down=True)

    def ew(e):
        return tuple(torch.from_numpy(oq3.dequant(b.data[e].cpu().numpy().view(np.uint32), b.scales[e].cpu().numpy(),
                                                  b.biases[e].cpu().numpy()))
                     for b in (layer.w1, layer.w3, layer.w2))
    ref = omoe.moe_combine(x, ids.long(), w.float(), ew, shared=None, limit=10.0)
    assert rel_l2(got, ref) <= TOL


def test_q3_medium_zipf_with_dropped_slots(cuda):
    got, ref, *_ = run_case(cuda, 1024, 512, 32, 4, 300, 10.0, True, seed=12, zipf=True, drop=0.1, fmt="q3")
    assert rel_l2(got, ref) <= TOL


def test_q3_config4_size(cuda):
    """Config-4 shapes over q3 banks: 2048 tokens, hidden 4096, 256 experts
    (inter 2048), top-8 Zipf(1.1); deterministic."""
    got, ref, ffn, x, ids, w = run_case(cuda, 4096, 2048, 256, 8, 2048, 10.0, True, seed=4, zipf=True, fmt="q3")
    assert rel_l2(got, ref) <= TOL
    again = ffn(x, ids, w.float(), route_before_down=True)
    assert torch.equal(again, got), "grouped path must be deterministic"


def test_q3_matches_decode_path(cuda):
    """Same q3 layer through the q3 decode kernels (validated against the CPU oracle)."""
    layer = synthetic.make_layer("q3", 4096, 2048, 64, seed=21, shared_inter=None, device=cuda)
    g = torch.Generator(device=cuda).manual_seed(21)
    x = torch.randn(8, 4096, generator=g, device=cuda).to(torch.bfloat16)
    w, ids = omoe.route_softmax_topk(torch.randn(8, 64, generator=g, device=cuda), 8)
    ids = ids.to(torch.int32)
    got = grouped.GroupedFFN(layer, 8)(x, ids, w.float(), route_before_down=True)
    dec = moe.moe_decode(x, layer, ids, w.float())
    assert rel_l2(got, dec) <= TOL


def test_q3_out_of_range_expert_gives_nan_not_fault(cuda):
    layer = synthetic.make_layer("q3", 256, 256, 8, seed=5, shared_inter=None, device=cuda)
    x = torch.randn(4, 256, device=cuda).to(torch.bfloat16)
    ids = torch.tensor([[0, 1], [2, 9], [3, 4], [5, 6]], dtype=torch.int32, device=cuda)
    w = torch.full((4, 2), 0.5, device=cuda)
    out = grouped.GroupedFFN(layer, 2)(x, ids, w)
    torch.cuda.synchronize()
    assert torch.isnan(out.float()).all()
