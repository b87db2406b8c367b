"""Router kernel vs the oracle (mlx_forward.py:62-81 and BASELINE's softmax top-k)."""
from __future__ import annotations

import pytest
import torch

from deepseeker import moe
from oracle import moe as omoe

pytestmark = pytest.mark.gpu


def pairs(idx, w):
    return sorted(zip(idx.flatten().tolist(), w.flatten().tolist()))


def test_router_matches_torch_gate(cuda):
    # tests/test_mlx_numerics.py:69-89
    torch.manual_seed(2)
    n, dim, n_exp, top_k = 3, 16, 8, 2
    x = torch.randn(n, dim)
    w = torch.randn(n_exp, dim) * 0.1
    b = torch.randn(n_exp)
    scores = torch.sqrt(torch.nn.functional.softplus(x @ w.T))
    indices = (scores + b).topk(top_k, dim=-1)[1]
    weights = scores.gather(1, indices)
    weights = weights / (weights.sum(-1, keepdim=True) + 1e-20) * 1.5
    gw, gidx = moe.route_topk(moe.sqrtsoftplus_scores(x.cuda(), w.cuda()), b.cuda(), top_k)
    got, want = pairs(gidx.cpu(), gw.cpu()), pairs(indices, weights)
    assert [p[0] for p in got] == [p[0] for p in want]
    torch.testing.assert_close(torch.tensor([p[1] for p in got]), torch.tensor([p[1] for p in want]),
                               rtol=1e-4, atol=1e-4)
    # fused logits -> sqrt-softplus -> top-k path
    fw, fidx = moe.route_sqrtsoftplus((x @ w.T).cuda(), b.cuda(), top_k)
    assert pairs(fidx.cpu(), fw.cpu())[0][0] == got[0][0]
    torch.testing.assert_close(fw.cpu(), gw.cpu(), rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("k", [2, 3, 4, 6])
def test_route_topk_narrow_k_keeps_per_row_sum(k, cuda):
    # tests/test_batch.py:320-337
    g = torch.Generator().manual_seed(1)
    scores = torch.randn(5, 384, generator=g) * 0.05 + 0.4
    w, idx = moe.route_topk(scores.cuda(), torch.zeros(384).cuda(), k)
    idx = idx.cpu()
    assert idx.shape == (5, k) and int(idx.min()) >= 0 and int(idx.max()) < 384
    for row in range(5):
        assert len(set(idx[row].tolist())) == k
        assert abs(float(w[row].sum()) - 1.5) < 1e-4
    ow, oidx = omoe.route_topk(scores, torch.zeros(384), k)
    assert sorted(oidx.flatten().tolist()) == sorted(idx.flatten().tolist())


def test_softmax_topk_matches_oracle(cuda):
    g = torch.Generator().manual_seed(3)
    logits = torch.randn(16, 256, generator=g)
    w, idx = moe.route_softmax_topk(logits.cuda(), 8)
    ow, oidx = omoe.route_softmax_topk(logits, 8)
    assert torch.equal(idx.cpu().long(), oidx)
    torch.testing.assert_close(w.cpu(), ow, rtol=1e-5, atol=1e-7)
    # ties go to the lower id
    t = torch.zeros(1, 64)
    w, idx = moe.route_softmax_topk(t.cuda(), 4)
    assert idx.cpu().tolist() == [[0, 1, 2, 3]]
    torch.testing.assert_close(w.cpu(), torch.full((1, 4), 0.25))
