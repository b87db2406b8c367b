"""moe.DecodeGraph: router + decode captured into a CUDA graph must give the
same output as the eager calls on the same inputs (bit for bit)."""
from __future__ import annotations

import pytest
import torch

from deepseeker import moe, synthetic

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("prepared", [True, False])
def test_graph_replay_matches_eager(prepared, cuda):
    layer = synthetic.make_layer("fp4", 4096, 2048, 64, seed=33, shared_inter=2048, device=cuda)
    if prepared:
        layer.prepare_tc()
    g = moe.DecodeGraph(layer, 1, 8)
    for step in range(3):
        x = torch.randn(1, 4096, device=cuda).to(torch.bfloat16)
        logits = torch.randn(1, 64, device=cuda)
        g.x.copy_(x)
        g.logits.copy_(logits)
        got = g.replay().clone()
        w, ids = moe.route_softmax_topk(logits, 8)
        ref = moe.moe_decode(x, layer, ids, w)
        torch.cuda.synchronize()
        assert torch.equal(got, ref), step


@pytest.mark.parametrize("in_place", [True, False])
def test_graph_chain_matches_eager(in_place, cuda):
    """Three layers in one graph (GraphChain): each layer's output equals the
    eager router + decode on its own inputs, with the staged inputs read in
    place or copied into the layers' buffers inside the graph."""
    layers = [synthetic.make_layer("fp4", 4096, 2048, 64, seed=40 + i, shared_inter=2048, device=cuda).prepare_tc()
              for i in range(3)]
    T = 2
    if in_place:
        sx = torch.zeros(3, T, 4096, dtype=torch.bfloat16, device=cuda)
        sl = torch.zeros(3, T, 64, device=cuda)
        graphs = [moe.DecodeGraph(l, T, 8, x=sx[i], logits=sl[i]) for i, l in enumerate(layers)]
        chain = moe.GraphChain(graphs, x=sx, logits=sl)
    else:
        graphs = [moe.DecodeGraph(l, T, 8) for l in layers]
        chain = moe.GraphChain(graphs)
    for step in range(2):
        xs = torch.randn(3, T, 4096, device=cuda).to(torch.bfloat16)
        lg = torch.randn(3, T, 64, device=cuda)
        chain.x.copy_(xs)
        chain.logits.copy_(lg)
        chain.replay()
        for i, l in enumerate(layers):
            w, ids = moe.route_softmax_topk(lg[i], 8)
            ref = moe.moe_decode(xs[i].contiguous(), l, ids, w)
            torch.cuda.synchronize()
            assert torch.equal(graphs[i].out, ref), (step, i)


def test_graph_chain_rejects_foreign_buffers(cuda):
    layer = synthetic.make_layer("fp4", 1024, 1024, 16, seed=1, device=cuda)
    g = moe.DecodeGraph(layer, 1, 4)
    with pytest.raises(ValueError):
        moe.GraphChain([g], x=torch.zeros(1, 1, 1024, dtype=torch.bfloat16, device=cuda),
                       logits=torch.zeros(1, 1, 16, device=cuda))


@pytest.mark.parametrize("fmt,atoms,T", [("fp4", True, 1), ("fp4", True, 3), ("fp4", False, 1), ("q3", False, 2)])
def test_graph_host_io_matches_eager(fmt, atoms, T, cuda):
    """host_io: pinned host in (staging kernel), one graph launch, the layer's
    output rows written straight into pinned host memory; every decode path
    (tcgen05, single-token register dequant, q3) gives the device path's bits."""
    layer = synthetic.make_layer(fmt, 4096, 2048, 64, seed=35, shared_inter=2048, device=cuda)
    if atoms:
        layer.prepare_tc()
    g = moe.DecodeGraph(layer, T, 8, host_io=True)
    for step in range(3):
        x = torch.randn(T, 4096).to(torch.bfloat16)
        logits = torch.randn(T, 64)
        g.x_host.copy_(x)
        g.logits_host.copy_(logits)
        got = g.replay_host().clone()
        w, ids = moe.route_softmax_topk(logits.to(cuda), 8)
        ref = moe.moe_decode(x.to(cuda), layer, ids, w).cpu()
        assert torch.equal(got, ref), step


def test_routed_call_writes_pinned_host_output(cuda):
    layer = synthetic.make_layer("fp4", 4096, 2048, 64, seed=36, shared_inter=2048, device=cuda).prepare_tc()
    x = torch.randn(2, 4096, device=cuda).to(torch.bfloat16)
    logits = torch.randn(2, 64, device=cuda)
    ref, _ = moe.moe_decode_routed(x, layer, logits, 8)
    host = torch.zeros(2, 4096, dtype=torch.bfloat16).pin_memory()
    out, _ = moe.moe_decode_routed(x, layer, logits, 8, out=host)
    moe.wait_stream(cuda)
    assert out is host and torch.equal(host, ref.cpu())
    with pytest.raises(ValueError):                 # pageable memory has no device mapping
        moe.moe_decode_routed(x, layer, logits, 8, out=torch.zeros(2, 4096, dtype=torch.bfloat16))
