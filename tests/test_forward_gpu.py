"""The mlx_forward MoE surface of the drop-in (``deepseeker.moe``): qmm,
gate/up stacking, the banked gather, the read-pipeline hooks and
``moe_layer`` with the reference's (expert_fn, shared_fn) contract.

Equalities restated from the reference's tests/test_mlx_forward.py:42-90,
128-158, 241-321 (MLX's quantiser replaced by the oracle's FP4 quantiser);
numerics against the torch fp32 oracle (oracle.moe, the restatement of
mlx_forward.py:84-103 and 388-419) at relative L2 <= 1e-3 (1e-5 where the
whole computation is f32).
"""
from __future__ import annotations

from concurrent.futures import Future

import numpy as np
import pytest
import torch

from deepseeker import moe, synthetic
from oracle import fp4 as ofp4
from oracle import moe as omoe
from oracle import q3 as oq3
from tests.test_decode_gpu import TOL, dense_expert, oracle_out, rel_l2

pytestmark = pytest.mark.gpu


def fp4_operands(n, k, seed, scale=1.0, device="cuda"):
    """(packed u8 [n, k/2], scales u8 [n, k/32]) of N(0, scale) weights, and the dense f32 matrix."""
    w = (torch.randn(n, k, generator=torch.Generator().manual_seed(seed)) * scale).numpy()
    p, s = ofp4.quantize_fp4(w)
    dense = torch.from_numpy(ofp4.dequant_matrix(p, s))
    return (torch.from_numpy(p).to(device), torch.from_numpy(s).to(device)), dense


def q3_operands(n, k, seed, scale=0.05, device="cuda"):
    w = (torch.randn(n, k, generator=torch.Generator().manual_seed(seed)) * scale).numpy()
    words, sc, bi = oq3.quantize(w)
    dense = torch.from_numpy(oq3.dequant(words, sc, bi))
    return ((torch.from_numpy(words.view(np.int32)).to(device), torch.from_numpy(sc).to(device),
             torch.from_numpy(bi).to(device)), dense)


@pytest.mark.parametrize("fmt", ["fp4", "q3"])
@pytest.mark.parametrize("rows", [1, 3, 8, 11])
@pytest.mark.parametrize("xdt", [torch.float32, torch.bfloat16])
def test_qmm_matches_oracle(fmt, rows, xdt, cuda):
    ops, dense = (fp4_operands if fmt == "fp4" else q3_operands)(96, 512, seed=rows)
    x = torch.randn(rows, 512, generator=torch.Generator().manual_seed(9)).to(xdt)
    got = moe.qmm(x.cuda(), ops)
    assert got.dtype == torch.float32 and got.shape == (rows, 96)
    ref = x.float() @ dense.T
    assert rel_l2(got, ref) < 1e-5


def test_qmm_accepts_the_u32_word_view(cuda):
    (p, s), dense = fp4_operands(64, 256, seed=2)
    x = torch.randn(2, 256, device=cuda)
    a = moe.qmm(x, (p, s))
    b = moe.qmm(x, (p.view(torch.int32), s))
    assert torch.equal(a, b)


def test_gate_up_stack_roundtrip_preserves_single_row_qmm_exactly(cuda):
    """Stacked w13 reproduces the separate w1 / w3 single-row outputs bit for bit."""
    x = torch.randn(1, 64, generator=torch.Generator().manual_seed(73)).cuda()
    w1, _ = fp4_operands(32, 64, seed=1)
    w3, _ = fp4_operands(32, 64, seed=2)
    expert = moe.stack_gate_up_expert({"w1": w1, "w3": w3, "w2": w1})
    split = moe.split_gate_up_expert(expert)
    expected = (moe.qmm(x, w1), moe.qmm(x, w3))
    actual = torch.chunk(moe.qmm(x, expert["w13"]), 2, dim=-1)
    assert torch.equal(actual[0], expected[0]) and torch.equal(actual[1], expected[1])
    assert torch.equal(moe.qmm(x, split["w1"]), expected[0])
    assert torch.equal(moe.qmm(x, split["w3"]), expected[1])
    with pytest.raises(ValueError):
        moe.stack_gate_up_expert({"w1": w1, "w3": w3[:1], "w2": w1})


def _bank(n_exp, dim, mid, seed, scale=0.1):
    return {e: (fp4_operands(mid, dim, seed * 100 + 3 * e, scale)[0],
                fp4_operands(mid, dim, seed * 100 + 3 * e + 1, scale)[0],
                fp4_operands(dim, mid, seed * 100 + 3 * e + 2, scale)[0]) for e in range(n_exp)}


def test_stacked_gate_up_preserves_single_and_multirow_moe_outputs(cuda):
    dim, mid, n_exp, top_k = 64, 32, 8, 2
    bank = _bank(n_exp, dim, mid, seed=91)
    stacked = {e: moe.stack_gate_up_expert({"w1": b[0], "w3": b[1], "w2": b[2]}) for e, b in bank.items()}
    g = torch.Generator().manual_seed(91)
    gate_w = torch.randn(n_exp, dim, generator=g).cuda()
    gate_b = torch.zeros(n_exp, device=cuda)
    for rows in (1, 3):
        x = torch.randn(rows, dim, generator=g).cuda()
        expected = moe.moe_layer(x, gate_w, gate_b, lambda e: bank[e], None, top_k)
        actual = moe.moe_layer(x, gate_w, gate_b, lambda e: stacked[e], None, top_k, stack_gateup=True)
        assert torch.equal(actual, expected)


def test_pipeline_hooks_give_the_plain_result(cuda):
    dim, mid, n_exp, top_k = 64, 32, 8, 2
    bank = _bank(n_exp, dim, mid, seed=121)
    g = torch.Generator().manual_seed(121)
    x = torch.randn(1, dim, generator=g).cuda()
    gate_w = torch.randn(n_exp, dim, generator=g).cuda()
    gate_b = torch.zeros(n_exp, device=cuda)
    expected = moe.moe_layer(x, gate_w, gate_b, lambda e: bank[e], None, top_k)
    finalized = []

    def submit(_layer, expert):
        fut = Future()
        w1, w3, w2 = bank[expert]
        fut.set_result(({"w1": w1, "w3": w3, "w2": w2}, 0, False, 0.0, 0.0))
        return fut

    actual = moe.moe_layer(x, gate_w, gate_b, lambda e: bank[e], None, top_k, pipeline=True,
                           async_submit_fn=submit, async_finalize_fn=lambda *a: finalized.append(a),
                           stack_gateup=True)
    assert torch.equal(actual, expected)
    assert len(finalized) == 1 and sorted(finalized[0][1]) == finalized[0][1]


def test_moe_layer_shapes_trace_and_prefetch(cuda):
    dim, mid, n_exp, top_k = 64, 32, 8, 2
    bank = _bank(n_exp, dim, mid, seed=3)
    g = torch.Generator().manual_seed(3)
    x = torch.randn(3, dim, generator=g).cuda()
    gate_w = (torch.randn(n_exp, dim, generator=g) * 0.1).cuda()
    gate_b = torch.zeros(n_exp, device=cuda)
    seen, fetched = [], []
    out = moe.moe_layer(x, gate_w, gate_b, lambda e: bank[e], lambda t: torch.zeros_like(t), top_k,
                        trace_hook=lambda layer, idx, w: seen.append((layer, idx, w)), layer_id=5,
                        prefetch_fn=lambda layer, experts: fetched.append((layer, experts)))
    assert out.shape == (3, dim)
    assert len(seen) == 1 and seen[0][0] == 5
    assert np.asarray(seen[0][1]).shape == (3, top_k)
    # slots in ascending biased-score order, as the reference's argsort gives
    scores = omoe.sqrtsoftplus_scores(x.cpu(), gate_w.cpu())
    for r, row in enumerate(seen[0][1]):
        assert scores[r, row[0]] <= scores[r, row[1]]
    assert fetched == [(5, sorted({e for row in seen[0][1] for e in row}))]


def test_banked_pins_match_serial_expert_path(cuda):
    dim, mid, n_exp, top_k = 64, 32, 8, 3
    bank = _bank(n_exp, dim, mid, seed=31)
    g = torch.Generator().manual_seed(31)
    x = torch.randn(4, dim, generator=g).cuda()
    gate_w = (torch.randn(n_exp, dim, generator=g) * 0.1).cuda()
    gate_b = (torch.randn(n_exp, generator=g) * 0.01).cuda()
    pins = [0, 2, 3, 6]
    slots = {e: i for i, e in enumerate(pins)}
    banks = {role: tuple(torch.stack([bank[e][ri][j] for e in pins]) for j in range(2))
             for role, ri in (("w1", 0), ("w2", 2), ("w3", 1))}
    plain = moe.moe_layer(x, gate_w, gate_b, lambda e: bank[e], None, top_k)

    def pinned_fn(layer, activations, indices, weights):
        return moe.gather_pinned_contributions(activations, indices, weights, banks, slots)

    banked = moe.moe_layer(x, gate_w, gate_b, lambda e: bank[e], None, top_k, pinned_gather_fn=pinned_fn)
    assert torch.allclose(plain, banked, atol=1e-6, rtol=1e-5)


def test_router_bias_steers_and_scores_are_positive(cuda):
    scores = (torch.randn(2, 8, generator=torch.Generator().manual_seed(0)) * 0.01 + 0.5).cuda()
    bias = torch.tensor([0, 0, 0, 0, 0, 0, 0, 10.0], device=cuda)
    w, idx = moe.route_topk(scores, bias, 2)
    assert 7 in idx[0].tolist()
    assert abs(float(w[0].sum()) - 1.5) < 1e-4
    s = moe.sqrtsoftplus_scores(torch.tensor([[-100.0, 0.0, 100.0]], device=cuda), torch.eye(3, device=cuda))
    assert bool((s >= 0).all())


@pytest.mark.parametrize("xdt", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("fmt", ["fp4", "q3"])
def test_moe_layer_resident_callable_and_oracle_agree(xdt, fmt, cuda):
    """Resident banks (fused kernels), the same banks through per-expert qmm
    callables, and the oracle: all within the decode tolerance; f32
    activations are not rounded to bf16 on the way (the reference runs the
    experts on x.astype(f32), mlx_forward.py:397)."""
    H, I, E, k = 1024, 512, 16, 4
    layer = synthetic.make_layer(fmt, H, I, E, seed=12, shared_inter=512, std=0.05)
    g = torch.Generator().manual_seed(12)
    x = torch.randn(3, H, generator=g).to(xdt)
    gate_w = torch.randn(E, H, generator=g) * 0.02
    gate_b = torch.randn(E, generator=g) * 0.01
    fused = moe.moe_layer(x.cuda(), gate_w.cuda(), gate_b.cuda(), layer.resident(), layer.shared_expert(), k)
    res = layer.resident()
    per_expert = moe.moe_layer(x.cuda(), gate_w.cuda(), gate_b.cuda(), lambda e: res(e), layer.shared_expert(), k)
    assert fused.dtype == xdt and per_expert.dtype == xdt
    scores = omoe.sqrtsoftplus_scores(x, gate_w)
    wts, idx = omoe.route_topk(scores, gate_b, k)
    ref = oracle_out(x, idx.to(torch.int32), wts, layer, 10.0)
    assert rel_l2(fused, ref) < TOL
    assert rel_l2(per_expert, ref) < TOL
    if xdt == torch.float32:
        # every step in f32: far inside the bar, and the bf16-rounded x would not be
        xb = x.to(torch.bfloat16).float()
        ref_b = oracle_out(xb, idx.to(torch.int32), wts, layer, 10.0)
        assert rel_l2(fused, ref) < 1e-5
        assert rel_l2(ref_b, ref) > 10 * rel_l2(fused, ref)


def test_moe_layer_without_shared_and_with_a_foreign_shared_fn(cuda):
    H, I, E, k = 1024, 1024, 8, 2
    layer = synthetic.make_layer("fp4", H, I, E, seed=5, shared_inter=1024, std=0.05)
    g = torch.Generator().manual_seed(5)
    x = torch.randn(1, H, generator=g).to(torch.bfloat16)
    gate_w = torch.randn(E, H, generator=g) * 0.02
    gate_b = torch.zeros(E)
    scores = omoe.sqrtsoftplus_scores(x, gate_w)
    wts, idx = omoe.route_topk(scores, gate_b, k)
    routed = synthetic.make_layer("fp4", H, I, E, seed=5, shared_inter=None, std=0.05)
    ref_no_shared = oracle_out(x, idx.to(torch.int32), wts, routed, 10.0)
    out = moe.moe_layer(x.cuda(), gate_w.cuda(), gate_b.cuda(), layer.resident(), None, k)
    assert rel_l2(out, ref_no_shared) < TOL
    # an arbitrary callable as shared_fn: added to the unrounded routed sum
    sh = layer.shared_expert()
    out2 = moe.moe_layer(x.cuda(), gate_w.cuda(), gate_b.cuda(), layer.resident(), lambda t: sh(t), k)
    ref = oracle_out(x, idx.to(torch.int32), wts, layer, 10.0)
    assert rel_l2(out2, ref) < TOL
