"""FP4 throughput mode of the grouped FFN (ds_grouped_ffn_fp4): FP4 banks
times activations rounded to FP4 (one e2m1 value per element, per-32 ue8m0
scale mapping the block maximum into (3, 6]), kind::mxf4 MMAs.

Its contract is the layer evaluated on the FP4-rounded x and h, so the
reference here is an emulation that rounds x and h the same way (the scale
rule, round-to-nearest-even onto the e2m1 grid) around float64 products with
the bit-exact dequantised weights (mlx_forward.py:388-419 semantics).
Tolerance against the emulation: relative L2 <= 5e-3 (f32 accumulation
order, and an element of h that lands on a rounding boundary can round the
other way); against the exact layer it is reported (of order 0.1), not
bounded tightly.
"""
from __future__ import annotations

import pytest
import torch

from deepseeker import grouped, metal_fp4, synthetic
from oracle import moe as omoe

pytestmark = pytest.mark.gpu

GRID = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)


def rel_l2(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def round_e2m1(v: torch.Tensor) -> torch.Tensor:
    """Round to nearest e2m1 value, ties to the even code, saturating at 6."""
    grid = torch.tensor(GRID, dtype=v.dtype, device=v.device)
    mids = (grid[1:] + grid[:-1]) / 2
    a = v.abs()
    idx = (a.unsqueeze(-1) > mids).sum(-1)
    tie = (a.unsqueeze(-1) == mids).any(-1) & (idx % 2 == 1)
    idx = torch.where(tie, idx + 1, idx).clamp(max=7)
    return torch.sign(v) * grid[idx]


def fp4_round_blocks(v: torch.Tensor) -> torch.Tensor:
    """v [..., n] f32, n % 32 == 0 -> each 32-block rounded to FP4 with the kernel's scale rule."""
    shp = v.shape
    b = v.reshape(-1, 32).float()
    amax = b.abs().amax(-1)
    bits = amax.view(torch.int32)
    ef = (bits >> 23) & 0xFF
    s = torch.where((bits & 0x7FFFFF) <= 0x400000, ef - 2, ef - 1).clamp(1, 253)
    s = torch.where(ef == 0, torch.full_like(s, 127), s)
    scale = torch.exp2((s - 127).double()).float()
    inv = torch.exp2((127 - s).double()).float()
    q = round_e2m1(b * inv[:, None]) * scale[:, None]
    return q.reshape(shp)


def emulate(x, layer, ids, w, limit, before):
    """Layer on FP4-rounded x and h, float64 products, result as the kernel combines it."""
    T, H = x.shape
    I = layer.inter
    xq = fp4_round_blocks(x.float())
    out = torch.zeros(T, H, dtype=torch.float64, device=x.device)
    for e in torch.unique(ids[ids >= 0]).tolist():
        rows, slots = torch.nonzero(ids == e, as_tuple=True)
        w1 = metal_fp4.dequant(layer.w1.data[e], layer.w1.scales[e]).view(I, H).double()
        w3 = metal_fp4.dequant(layer.w3.data[e], layer.w3.scales[e]).view(I, H).double()
        w2 = metal_fp4.dequant(layer.w2.data[e], layer.w2.scales[e]).view(H, I).double()
        xr = xq[rows].double()
        g, u = xr @ w1.T, xr @ w3.T
        if limit:
            g, u = g.clamp(max=limit), u.clamp(-limit, limit)
        h = g / (1 + torch.exp(-g)) * u
        gw = w[rows, slots].double()[:, None]
        if before:
            h = h * gw
        hq = fp4_round_blocks(h.float()).double()
        y = hq @ w2.T
        if not before:
            y = y * gw
        out.index_add_(0, rows, y)
    return out


def exact(x, layer, ids, w, limit, before):
    from tests.test_grouped_gpu import torch_reference
    return torch_reference(x, layer, ids, w, limit, before)


def test_round_e2m1_ties_to_even():
    v = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 7.0, -0.75, 0.3])
    assert round_e2m1(v).tolist() == [0.0, 1.0, 1.0, 2.0, 2.0, 4.0, 4.0, 6.0, -1.0, 0.5]


@pytest.mark.parametrize("before,limit", [(True, 10.0), (False, None)])
def test_fp4_activations_small(before, limit, cuda):
    H, I, E, k, T = 512, 256, 8, 2, 37
    layer = synthetic.make_layer("fp4", H, I, E, seed=11, shared_inter=None, device=cuda, limit=limit)
    g = torch.Generator(device=cuda).manual_seed(11)
    x = torch.randn(T, H, generator=g, device=cuda).to(torch.bfloat16)
    wts, ids = omoe.route_softmax_topk(torch.randn(T, E, generator=g, device=cuda), k)
    ids, wts = ids.to(torch.int32), wts.float()
    got = grouped.GroupedFFN(layer, k, activations="fp4")(x, ids, wts, route_before_down=before,
                                                          out_dtype=torch.float32)
    emu = emulate(x, layer, ids, wts, limit, before)
    assert torch.isfinite(got).all()
    assert rel_l2(got, emu) <= 5e-3, rel_l2(got, emu)
    assert rel_l2(got, exact(x, layer, ids, wts, limit, before)) <= 0.3


def test_fp4_activations_config4_size(cuda):
    """2048 tokens, hidden 4096, 256 experts (inter 2048), top-8 Zipf(1.1)."""
    H, I, E, k, T = 4096, 2048, 256, 8, 2048
    layer = synthetic.make_layer("fp4", H, I, E, seed=4, shared_inter=None, device=cuda)
    g = torch.Generator(device=cuda).manual_seed(4)
    x = torch.randn(T, H, generator=g, device=cuda).to(torch.bfloat16)
    ids, wts = synthetic.zipf_routing(T, E, k, seed=4, device=cuda)
    ffn = grouped.GroupedFFN(layer, k, activations="fp4")
    got = ffn(x, ids, wts, route_before_down=True, out_dtype=torch.float32)
    emu = emulate(x, layer, ids, wts, 10.0, True)
    assert rel_l2(got, emu) <= 5e-3, rel_l2(got, emu)
    again = ffn(x, ids, wts, route_before_down=True, out_dtype=torch.float32)
    assert torch.equal(got, again), "deterministic"


def test_fp4_activations_needs_fp4_banks(cuda):
    layer = synthetic.make_layer("q3", 256, 256, 4, seed=1, shared_inter=None, device=cuda)
    with pytest.raises(NotImplementedError):
        grouped.GroupedFFN(layer, 2, activations="fp4")
