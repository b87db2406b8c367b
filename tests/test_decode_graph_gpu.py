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
