"""Router + decode layer in one call (ds_moe_decode_route).

On the tcgen05 kernels the prep kernel routes the tokens itself, one warp
per token, in the router kernel's reduction order: its ids and gates must
equal ds_route_topk's bit for bit (softmax, sqrt-softplus with bias, raw
scores; ties, NaN logits, 64..520 experts), and the layer output must equal
route_* followed by moe_decode bit for bit.  Other kernels route first in
their own launch (same contract).  The routed output is also checked against
the CPU oracle's routing + layer (mlx_forward.py:62-81, 388-419).
"""
from __future__ import annotations

import pytest
import torch

from deepseeker import moe, synthetic
from oracle import moe as omoe
from tests.test_decode_gpu import TOL, oracle_out, rel_l2

pytestmark = pytest.mark.gpu

_LAYERS: dict = {}


def layer_of(E, k, tc=True, fmt="fp4"):
    key = (E, tc, fmt)
    if key not in _LAYERS:
        layer = synthetic.make_layer(fmt, 1024, 1024, E, seed=300 + E, shared_inter=256, std=0.05, limit=10.0)
        _LAYERS[key] = layer.prepare_tc() if tc else layer
    return _LAYERS[key]


def two_calls(x, layer, logits, k, kind, bias, scale):
    if kind == "softmax":
        w, ids = moe.route_softmax_topk(logits, k)
    elif kind == "sqrtsoftplus":
        w, ids = moe.route_sqrtsoftplus(logits, bias, k, route_scale=scale)
    else:
        w, ids = moe.route_topk(logits, bias, k, route_scale=scale)
    return moe.moe_decode(x, layer, ids, w), w, ids


def make_logits(T, E, seed, ties=False, nan=False):
    g = torch.Generator().manual_seed(seed)
    lg = torch.randn(T, E, generator=g) * 2
    if ties:
        lg = torch.round(lg)            # many equal keys
    if nan:
        lg[0, 3] = float("nan")
        lg[-1, E // 2] = float("nan")
    return lg


@pytest.mark.parametrize("E", [64, 256, 384, 520])
@pytest.mark.parametrize("kind", ["softmax", "sqrtsoftplus", "scores"])
def test_fused_routing_bit_identical(E, kind, cuda):
    k = 8
    layer = layer_of(E, k)
    bias = (torch.randn(E, generator=torch.Generator().manual_seed(E)) * 0.1).cuda() if kind != "softmax" else None
    for T, ties, nan in ((1, False, False), (3, True, False), (8, False, True), (8, True, True)):
        logits = make_logits(T, E, seed=E + T, ties=ties, nan=nan).cuda()
        x = torch.randn(T, 1024, generator=torch.Generator().manual_seed(T)).to(torch.bfloat16).cuda()
        out, (w, ids) = moe.moe_decode_routed(x, layer, logits, k, kind=kind, bias=bias, route_scale=1.5)
        ref, rw, rids = two_calls(x, layer, logits, k, kind, bias, 1.5)
        assert torch.equal(ids, rids), (E, kind, T)
        assert torch.equal(w.view(torch.int32), rw.view(torch.int32)), (E, kind, T)
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), (E, kind, T)


@pytest.mark.parametrize("tc,fmt", [(False, "fp4"), (False, "q3")])
def test_other_kernels_route_first(tc, fmt, cuda):
    E, k, T = 64, 6, 2
    layer = layer_of(E, k, tc=tc, fmt=fmt)
    logits = make_logits(T, E, seed=5).cuda()
    x = torch.randn(T, 1024, generator=torch.Generator().manual_seed(9)).to(torch.bfloat16).cuda()
    out, (w, ids) = moe.moe_decode_routed(x, layer, logits, k)
    ref, rw, rids = two_calls(x, layer, logits, k, "softmax", None, 1.0)
    assert torch.equal(ids, rids) and torch.equal(w, rw)
    assert torch.equal(out, ref)


@pytest.mark.parametrize("T", [1, 4])
def test_fused_routing_vs_oracle(T, cuda):
    E, k = 256, 8
    layer = layer_of(E, k)
    logits = make_logits(T, E, seed=70 + T)
    x = torch.randn(T, 1024, generator=torch.Generator().manual_seed(71)).to(torch.bfloat16)
    out, (w, ids) = moe.moe_decode_routed(x.cuda(), layer, logits.cuda(), k)
    ow, oids = omoe.route_softmax_topk(logits, k)
    assert torch.equal(ids.cpu().long(), oids.long())
    torch.testing.assert_close(w.cpu(), ow.float(), rtol=1e-5, atol=1e-7)
    assert rel_l2(out, oracle_out(x, oids.int(), ow.float(), layer, 10.0)) < TOL


def test_decode_graph_uses_routed_call(cuda):
    """DecodeGraph (one CUDA graph per layer) replays the routed call; the
    routing it leaves in .ids / .w equals the router's."""
    E, k, T = 256, 8, 2
    layer = layer_of(E, k)
    gr = moe.DecodeGraph(layer, T, k)
    logits = make_logits(T, E, seed=3).cuda()
    x = torch.randn(T, 1024, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16).cuda()
    gr.x.copy_(x)
    gr.logits.copy_(logits)
    out = gr.replay().clone()
    ref, rw, rids = two_calls(x, layer, logits, k, "softmax", None, 1.0)
    assert torch.equal(gr.ids, rids) and torch.equal(gr.w, rw)
    assert torch.equal(out, ref)
