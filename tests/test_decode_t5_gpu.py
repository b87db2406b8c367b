"""Decode layer on the tcgen05 kernels (FP4 banks with prepared scale atoms).

Checked against the CPU oracle (oracle.moe.moe_combine on the oracle's dense
dequant, the restatement of moe_layer's loop, mlx_forward.py:388-419) at
relative L2 <= 1e-3, and against the library's other decode kernels on the
same inputs (the same layer without scale atoms).
"""
from __future__ import annotations

import pytest
import torch

from deepseeker import moe, synthetic
from oracle import moe as omoe
from tests.test_decode_gpu import TOL, oracle_out, rel_l2, routing

pytestmark = pytest.mark.gpu


def t5_layer(H, I, E, seed, shared, limit=10.0, std=0.02):
    return synthetic.make_layer("fp4", H, I, E, seed=seed, shared_inter=shared, std=std, limit=limit).prepare_tc()


@pytest.mark.parametrize("T", [1, 3, 8])
def test_small_layer_vs_oracle(T, cuda):
    H, I, E, k = 1024, 1024, 16, 4
    layer = t5_layer(H, I, E, seed=40 + T, shared=256, std=0.05)
    ids, wts = routing(T, E, k, seed=T + 7)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(T)).to(torch.bfloat16)
    out = moe.moe_decode(x.cuda(), layer, ids.cuda(), wts.cuda())
    ref = oracle_out(x, ids, wts, layer, 10.0)
    assert out.dtype == torch.bfloat16 and out.shape == (T, H)
    assert rel_l2(out, ref) < TOL


def test_dropped_duplicate_and_no_shared(cuda):
    H, I, E, k = 1024, 1024, 8, 3
    layer = t5_layer(H, I, E, seed=51, shared=None, limit=None, std=0.1)
    ids = torch.tensor([[5, 2, 7], [1, -1, 5], [3, 3, 0]], dtype=torch.int32)
    wts = torch.tensor([[0.5, 0.3, 0.2], [0.6, 0.0, 0.4], [0.7, 0.1, 0.2]])
    x = (torch.randn(3, H, generator=torch.Generator().manual_seed(3)) * 2).to(torch.bfloat16)
    out = moe.moe_decode(x.cuda(), layer, ids.cuda(), wts.cuda())
    ref = oracle_out(x, ids, wts, layer, None)
    assert rel_l2(out, ref) < TOL


@pytest.mark.parametrize("T", [1, 4])
def test_config2_full_layer_vs_oracle(T, cuda):
    """BASELINE config 2 geometry: hidden 4096, 256 FP4 experts (inter 2048), top-8, bf16 shared."""
    H, I, E, k = 4096, 2048, 256, 8
    layer = t5_layer(H, I, E, seed=2, shared=2048)
    ids, wts = routing(T, E, k, seed=12)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(13)).to(torch.bfloat16)
    out = moe.moe_decode(x.cuda(), layer, ids.cuda(), wts.cuda())
    again = moe.moe_decode(x.cuda(), layer, ids.cuda(), wts.cuda())
    assert torch.equal(out, again), "tcgen05 decode must be deterministic"
    ref = oracle_out(x, ids, wts, layer, 10.0)
    assert rel_l2(out, ref) < TOL


def test_matches_previous_kernels(cuda):
    """The same layer with scale atoms (tcgen05 kernels) and without them
    (single-token FP4 kernels) agrees within the decode tolerance."""
    layer = synthetic.make_layer("fp4", 4096, 2048, 64, seed=9, shared_inter=2048)
    w, idx = omoe.route_softmax_topk(torch.randn(1, 64, generator=torch.Generator().manual_seed(3)), 8)
    ids, wts = idx.to(torch.int32).cuda(), w.cuda()
    x = torch.randn(1, 4096, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16).cuda()
    plain = moe.moe_decode(x, layer, ids, wts)
    layer.prepare_tc()
    t5 = moe.moe_decode(x, layer, ids, wts)
    assert rel_l2(t5, plain) < TOL
