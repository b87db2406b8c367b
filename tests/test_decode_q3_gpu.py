"""q3 decode kernels (csrc/moe_decode_q3.cu: bf16 x, 1..8 tokens, streaming
CUDA-core dot products) vs the torch fp32 oracle of moe_layer
(mlx_forward.py:388-419) with the q3 groups dequantised by oracle/q3.py.
Shapes are chosen so that ds_moe_decode takes this path (hidden, inter and
the shared inter multiples of 128).  Tolerance: relative L2 <= 1e-3 (the
north-star bar).  The path multiplies the 3-bit codes with int8 pieces of the
activations (hi + lo / 256 per 64-value group: ~15 significant bits relative
to the group maximum; x and h are each cut once), so an f32 output sits near
1e-4 of the oracle; those cases are held to 5e-4.
"""
from __future__ import annotations

import pytest
import torch

from deepseeker import moe, synthetic
from tests.test_decode_gpu import TOL, oracle_out, rel_l2, routing

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T", [1, 2, 3, 5, 8])
def test_q3_path_tokens(T, cuda):
    H, I, E, k = 512, 256, 16, 4
    layer = synthetic.make_layer("q3", H, I, E, seed=50 + T, shared_inter=256, std=0.05)
    ids, wts = routing(T, E, k, seed=60 + T)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(70 + T)).to(torch.bfloat16)
    out = moe.moe_decode(x.cuda(), layer, ids.cuda(), wts.cuda())
    ref = oracle_out(x, ids, wts, layer, 10.0)
    assert out.dtype == torch.bfloat16 and out.shape == (T, H)
    assert rel_l2(out, ref) < TOL, rel_l2(out, ref)
    again = moe.moe_decode(x.cuda(), layer, ids.cuda(), wts.cuda())
    assert torch.equal(out, again)


def test_q3_path_dropped_repeated_slots_f32_out(cuda):
    """Dropped slot (-1), an expert repeated within a token, two tokens sharing
    an expert, no clamp, no shared expert; f32 output (no final rounding)."""
    H, I, E, k = 256, 128, 8, 3
    layer = synthetic.make_layer("q3", H, I, E, seed=21, shared_inter=None, std=0.2, limit=None)
    ids = torch.tensor([[5, 2, 7], [1, -1, 5], [3, 3, 0]], dtype=torch.int32)
    wts = torch.tensor([[0.5, 0.3, 0.2], [0.6, 0.0, 0.4], [0.7, 0.1, 0.2]])
    x = (torch.randn(3, H, generator=torch.Generator().manual_seed(3)) * 4.0).to(torch.bfloat16)
    out = moe.moe_decode(x.cuda(), layer, ids.cuda(), wts.cuda(), out_f32=True)
    ref = oracle_out(x.float(), ids, wts, layer, None)
    assert out.dtype == torch.float32
    assert rel_l2(out, ref) < 5e-4, rel_l2(out, ref)


def test_q3_path_gate_after_down(cuda):
    """grouped_swiglu semantics: the gate multiplies the down output (grouped.py:50-53)."""
    H, I, E, k = 256, 128, 8, 2
    layer = synthetic.make_layer("q3", H, I, E, seed=8, shared_inter=None, std=0.1, limit=None)
    layer.route_before_down = False
    ids, wts = routing(2, E, k, seed=9)
    x = torch.randn(2, H, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    out = moe.moe_decode(x.cuda(), layer, ids.cuda(), wts.cuda(), out_f32=True)
    ref = oracle_out(x.float(), ids, wts, layer, None)
    assert rel_l2(out, ref) < 5e-4, rel_l2(out, ref)


def test_q3_path_expert_id_out_of_range_sets_error(cuda):
    """An id >= n_experts is dropped on the device and bit 1 of the
    workspace error word is set (no out-of-bounds read)."""
    H, I, E, k = 256, 128, 8, 2
    layer = synthetic.make_layer("q3", H, I, E, seed=4, shared_inter=128, std=0.05)
    ws = torch.zeros(layer.decode_workspace_bytes(1, k), dtype=torch.uint8, device="cuda")
    ids = torch.tensor([[3, 99]], dtype=torch.int32, device="cuda")
    wts = torch.tensor([[0.5, 0.5]], device="cuda")
    x = torch.randn(1, H, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16).cuda()
    out = moe.moe_decode(x, layer, ids, wts, workspace=ws)
    torch.cuda.synchronize()
    assert int(ws[:4].view(torch.int32)[0]) & 1
    # the dropped id behaves exactly like an empty routing entry
    same = moe.moe_decode(x, layer, torch.tensor([[3, -1]], dtype=torch.int32, device="cuda"), wts)
    assert torch.equal(out, same)
    # 256 bf16 outputs: a few one-ulp rounding flips (2^-8 relative each)
    # already reach 1e-3 rel-L2, so the oracle bound here is 2e-3
    ref = oracle_out(x, torch.tensor([[3, -1]], dtype=torch.int32), wts, layer, 10.0)
    assert rel_l2(out, ref) < 2e-3, rel_l2(out, ref)
