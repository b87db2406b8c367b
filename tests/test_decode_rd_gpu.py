"""Single-token decode on the register-dequant kernel (moe_decode_rd.cu):
FP4 banks, bf16 x, one token; against the CPU oracle (oracle.moe.moe_combine
on the oracle's dense dequant, mlx_forward.py:388-419) at relative L2 <=
1e-3, plus its own properties: deterministic, control words left at zero,
graph replays equal eager calls, dropped / duplicate / out-of-range slots."""
from __future__ import annotations

import pytest
import torch

from deepseeker import moe, synthetic
from tests.test_decode_gpu import TOL, oracle_out, rel_l2, routing

pytestmark = pytest.mark.gpu


def layer_rd(H, I, E, seed, shared, limit=10.0, std=0.02):
    return synthetic.make_layer("fp4", H, I, E, seed=seed, shared_inter=shared, std=std, limit=limit)


@pytest.mark.parametrize("std", [0.02, 0.05])
@pytest.mark.parametrize("H,I,E,k,Is", [(4096, 2048, 32, 8, 2048), (5120, 2304, 12, 6, 2304),
                                         (512, 128, 8, 2, 128), (1024, 384, 16, 4, None),
                                         (2048, 1024, 16, 4, 1024)])
def test_layer_vs_oracle(H, I, E, k, Is, std, cuda):
    layer = layer_rd(H, I, E, seed=H + I, shared=Is, std=std)
    ids, wts = routing(1, E, k, seed=3)
    x = torch.randn(1, H, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16)
    out = moe.moe_decode(x.cuda(), layer, ids.cuda(), wts.cuda())
    again = moe.moe_decode(x.cuda(), layer, ids.cuda(), wts.cuda())
    assert torch.equal(out, again), "the single-token kernel must be deterministic"
    ref = oracle_out(x, ids, wts, layer, 10.0)
    assert rel_l2(out, ref) < TOL


def test_f32_output(cuda):
    H, I, E, k = 2048, 1024, 16, 4
    layer = layer_rd(H, I, E, seed=8, shared=1024, std=0.05)
    ids, wts = routing(1, E, k, seed=9)
    x = torch.randn(1, H, generator=torch.Generator().manual_seed(10)).to(torch.bfloat16)
    out = moe.moe_decode(x.cuda(), layer, ids.cuda(), wts.cuda(), out_f32=True)
    assert out.dtype == torch.float32
    # f32 output = the bf16 output before its final rounding (the shared
    # expert's output is rounded to bf16 in both, as in the reference)
    bf = moe.moe_decode(x.cuda(), layer, ids.cuda(), wts.cuda())
    assert torch.equal(out.to(torch.bfloat16), bf)
    assert rel_l2(bf, oracle_out(x, ids, wts, layer, 10.0)) < TOL


def test_no_clamp_one_token_takes_the_tcgen05_kernels(cuda):
    """Without the SwiGLU clamp there is no bound for h, so one token of a
    layer with scale atoms runs on the tcgen05 kernels; f32 output too."""
    H, I, E, k = 2048, 1024, 16, 4
    layer = layer_rd(H, I, E, seed=8, shared=1024, limit=None, std=0.05).prepare_tc()
    ids, wts = routing(1, E, k, seed=9)
    x = torch.randn(1, H, generator=torch.Generator().manual_seed(10)).to(torch.bfloat16)
    bf = moe.moe_decode(x.cuda(), layer, ids.cuda(), wts.cuda())
    f32 = moe.moe_decode(x.cuda(), layer, ids.cuda(), wts.cuda(), out_f32=True)
    assert torch.equal(f32.to(torch.bfloat16), bf)
    assert rel_l2(bf, oracle_out(x, ids, wts, layer, None)) < TOL


def test_dropped_duplicate_and_out_of_range_slots(cuda):
    H, I, E = 1024, 512, 8
    layer = layer_rd(H, I, E, seed=21, shared=512, std=0.05)
    x = torch.randn(1, H, generator=torch.Generator().manual_seed(22)).to(torch.bfloat16).cuda()
    w = torch.tensor([[0.4, 0.3, 0.2, 0.1]], device=cuda)
    ws = torch.zeros(layer.decode_workspace_bytes(1, 4), dtype=torch.uint8, device=cuda)
    # -1 dropped; 5 twice: the first slot's gate counts (mlx_forward.py:394-396); 99 out of range
    ids = torch.tensor([[5, -1, 5, 99]], dtype=torch.int32, device=cuda)
    out = moe.moe_decode(x, layer, ids, w, workspace=ws)
    torch.cuda.synchronize()
    assert int(ws[:4].view(torch.int32)[0]) & 1
    ref = oracle_out(x.cpu(), torch.tensor([[5, -1, 5, -1]], dtype=torch.int32), w.cpu(), layer, 10.0)
    assert rel_l2(out, ref) < TOL
    # no routed expert at all: the shared expert alone
    none = moe.moe_decode(x, layer, torch.full((1, 4), -1, dtype=torch.int32, device=cuda), w)
    ref0 = oracle_out(x.cpu(), torch.full((1, 4), -1, dtype=torch.int32), w.cpu(), layer, 10.0)
    assert rel_l2(none, ref0) < TOL


def test_control_words_return_to_zero_and_graph_replay(cuda):
    H, I, E, k = 2048, 1024, 16, 4
    layer = layer_rd(H, I, E, seed=31, shared=1024)
    nbytes = layer.decode_workspace_bytes(1, k)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=cuda)
    ids, wts = routing(1, E, k, seed=32)
    ids, wts = ids.cuda(), wts.cuda()
    x = torch.randn(1, H, generator=torch.Generator().manual_seed(33)).to(torch.bfloat16).cuda()
    moe.moe_decode(x, layer, ids, wts, workspace=ws)
    for _ in range(3):
        moe.moe_decode(x, layer, ids, wts, workspace=ws)
    torch.cuda.synchronize()
    # error word, grid-barrier words and shared-task counters: all zero again
    assert int(ws[:4096].count_nonzero()) == 0
    g = moe.DecodeGraph(layer, 1, k, cuda)
    g.x.copy_(x)
    lg = torch.randn(1, E, generator=torch.Generator().manual_seed(34)).cuda()
    g.logits.copy_(lg)
    outs = [g.replay().clone() for _ in range(3)]
    w2, i2 = moe.route_softmax_topk(lg, k)
    eager = moe.moe_decode(x, layer, i2, w2)
    for o in outs:
        assert torch.equal(o, eager)


def test_shared_expert_keeps_its_clamp_without_a_routed_clamp_tcgen05(cuda):
    """With the routed clamp off, the shared expert still clamps at 10 on the
    tcgen05 kernels too (two tokens, FP4 banks with scale atoms)."""
    H, I, E, k = 1024, 1024, 16, 4
    layer = layer_rd(H, I, E, seed=8, shared=1024, limit=None, std=0.05).prepare_tc()
    ids, wts = routing(2, E, k, seed=9)
    x = torch.randn(2, H, generator=torch.Generator().manual_seed(10)).to(torch.bfloat16)
    out = moe.moe_decode(x.cuda(), layer, ids.cuda(), wts.cuda())
    assert rel_l2(out, oracle_out(x, ids, wts, layer, None)) < TOL
