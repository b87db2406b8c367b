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


def test_graph_host_io_matches_eager(cuda):
    """host_io: pinned host in, one graph launch (copies inside), pinned host out."""
    layer = synthetic.make_layer("fp4", 4096, 2048, 64, seed=35, shared_inter=2048, device=cuda).prepare_tc()
    g = moe.DecodeGraph(layer, 1, 8, host_io=True)
    for step in range(3):
        x = torch.randn(1, 4096).to(torch.bfloat16)
        logits = torch.randn(1, 64)
        g.x_host.copy_(x)
        g.logits_host.copy_(logits)
        got = g.replay_host().clone()
        w, ids = moe.route_softmax_topk(logits.to(cuda), 8)
        ref = moe.moe_decode(x.to(cuda), layer, ids, w).cpu()
        assert torch.equal(got, ref), step
