"""The CPU oracle is pinned to the reference's own outputs (golden vectors from
tests/golden/make_golden.py) before anything is compared against it."""
from __future__ import annotations

import hashlib
import json

import numpy as np
import pytest
import torch

from oracle import fp4 as ofp4
from oracle import moe as omoe
from oracle import q3 as oq3


def bits_equal(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    assert a.shape == b.shape
    same = (a.view(np.uint32) == b.view(np.uint32)) | (np.isnan(a) & np.isnan(b))
    assert same.all(), np.where(~same)[0][:8]


def test_tables(golden):
    bits_equal(ofp4.FP4_TABLE, golden["fp4_table"])
    bits_equal(ofp4.decode_u8m0(np.arange(256, dtype=np.uint8)), golden["u8m0_all"])
    bits_equal(ofp4.decode_scales_u8m0(bytes(range(256))), golden["u8m0_all_metal"])
    bits_equal(ofp4.E4M3_TABLE, golden["e4m3_table"])
    # tests/test_metal_fp4.py:35-41 spot values
    assert ofp4.FP4_TABLE[0x7] == 6.0 and ofp4.FP4_TABLE[0xF] == -6.0 and ofp4.FP4_TABLE[0x8] == 0.0
    assert not np.signbit(ofp4.FP4_TABLE[0x8])


def test_fp4_vectors(golden):
    bits_equal(ofp4.dequant_f32_scales(golden["fp4_seed3_packed"], golden["fp4_seed3_scales"]),
               golden["fp4_seed3_out"])
    bits_equal(golden["fp4_seed3_out"], golden["fp4_seed3_torch"])
    bits_equal(ofp4.dequant_u8_scales(golden["fp4_seed2_packed"], golden["fp4_seed2_raw_scales"]),
               golden["fp4_seed2_out"])
    bits_equal(ofp4.dequant_u8_scales(np.array([0x13], np.uint8), np.array([128], np.uint8)),
               golden["fp4_nibble_out"])
    # tests/test_q3.py:132-141: low nibble first, [TABLE[3], TABLE[1]] * 2
    np.testing.assert_array_equal(golden["fp4_nibble_out"], ofp4.FP4_TABLE[[3, 1]] * 2.0)
    bits_equal(ofp4.dequant_u8_scales(np.array([0x21, 0x9F, 0x78], np.uint8), np.array([130], np.uint8)),
               golden["fp4_tail_out"])


def test_fp4_exhaustive(golden):
    packed = np.tile(np.arange(256, dtype=np.uint8), 256)
    scales = np.repeat(np.arange(256, dtype=np.uint8), 16)
    with np.errstate(over="ignore"):
        out = ofp4.dequant_u8_scales(packed, scales)
    bits_equal(out, golden["fp4_exhaustive_out"])


def test_fp4_bench_seed9_hash(golden):
    rng = np.random.default_rng(9)
    packed = rng.integers(0, 256, size=(5120 * 2304) // 2, dtype=np.uint8)
    scales = np.exp2(rng.integers(-2, 3, size=(5120 * 2304) // 32).astype(np.float32))
    h = golden["_hashes"]
    assert hashlib.sha256(packed.tobytes()).hexdigest() + ":" + hashlib.sha256(scales.tobytes()).hexdigest() \
        == h["bench_fp4_seed9_inputs"]
    out = ofp4.dequant_f32_scales(packed, scales)
    assert hashlib.sha256(out.tobytes()).hexdigest() == h["bench_fp4_seed9_out"]


def test_fp8_block(golden):
    bits_equal(ofp4.dequant_fp8_block(golden["fp8_seed1_packed"], golden["fp8_seed1_scales"]),
               golden["fp8_seed1_out"])
    want = torch.frombuffer(bytearray(range(256)), dtype=torch.float8_e4m3fn).float().numpy()
    bits_equal(ofp4.E4M3_TABLE, want)


def test_align_vectors(golden):
    topk = np.array([[1, 2, 3], [0, 1, 3], [0, 2, 3], [0, 1, 2]])
    s, e, n = omoe.align_block_size(topk, 4, 4)
    np.testing.assert_array_equal(s, golden["align_doc_sorted"])
    np.testing.assert_array_equal(e, golden["align_doc_experts"])
    assert n == int(golden["align_doc_npad"][0]) == 16
    s, e, n = omoe.align_block_size(golden["align_rand_topk"], 16, 384)
    np.testing.assert_array_equal(s, golden["align_rand_sorted"])
    np.testing.assert_array_equal(e, golden["align_rand_experts"])
    assert n == int(golden["align_rand_npad"][0])
    with pytest.raises(ValueError):
        omoe.align_block_size(np.array([1, 2, 3]), 4, 4)
    with pytest.raises(ValueError):
        omoe.align_block_size(np.array([[0, 99]]), 4, 4)


def test_plan_groups_golden(golden):
    want = json.loads(golden["_hashes"]["plan_groups_golden"])
    got = omoe.plan_groups([[2, 0], [1, 2], [0, 0]], 3)
    assert {str(k): [list(p) for p in v] for k, v in got.items()} == want
    assert omoe.plan_groups([[], []], 3) == {}
    with pytest.raises(ValueError):
        omoe.plan_groups([[9]], 3)


def test_fp4_quantizer_roundtrip_and_ties():
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((8, 256)) * 0.02).astype(np.float32)
    p, s = ofp4.quantize_fp4(w)
    assert p.shape == (8, 128) and s.shape == (8, 8)
    deq = ofp4.dequant_matrix(p, s)
    assert np.all(np.abs(deq - w) <= np.repeat(ofp4.decode_u8m0(s), 32, axis=1) * 1.0 + 1e-12)
    # ties go to the even code: 0.25 -> 0, 0.75 -> 1.0, 1.25 -> 1.0, 1.75 -> 2.0, 2.5 -> 2, 3.5 -> 4, 5 -> 4
    t = np.zeros((1, 32), np.float32)
    t[0, :8] = [6.0, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0]
    p, s = ofp4.quantize_fp4(t)
    assert s[0, 0] == 127
    np.testing.assert_array_equal(ofp4.dequant_matrix(p, s)[0, :8], [6.0, 0.0, 1.0, 1.0, 2.0, 2.0, 4.0, 4.0])


def test_q3_layout_roundtrip_and_geometry():
    rng = np.random.default_rng(7)
    q = rng.integers(0, 8, size=(5, 192)).astype(np.uint8)
    np.testing.assert_array_equal(oq3.unpack_codes(oq3.pack_codes(q), 192), q)
    # tests/test_q3.py:89-105 geometry: 8 x 256 -> 24 words/row, 4 groups/row
    vals = (rng.standard_normal(8 * 256) * 0.05).astype(np.float32).reshape(8, 256)
    words, s, b = oq3.quantize(vals)
    assert words.shape == (8, 24) and s.shape == (8, 4) and b.shape == (8, 4)
    assert s.dtype == np.float16 and b.dtype == np.float16
    rt = oq3.dequant(words, s, b)
    rms = oq3.rel_rms(vals, rt)
    assert 0.0 < rms < 0.08
    # layout: element j of low word 0 sits at bits [2j, 2j+2), element 8+j at [16+2j, ...)
    one = np.zeros((1, 64), np.uint8)
    one[0, 9] = 7  # low word 0 upper half j=1 -> bits 18..19; high word 0 bit 16+1
    wds = oq3.pack_codes(one)
    assert wds[0, 0] == (3 << 18) and wds[0, 4] == (1 << 17)


def test_oracle_moe_matches_grouped_and_naive():
    g = torch.Generator().manual_seed(0)
    weights = {e: (torch.randn(16, 8, generator=g) * 0.1, torch.randn(16, 8, generator=g) * 0.1,
                   torch.randn(8, 16, generator=g) * 0.1) for e in range(4)}
    x = torch.randn(5, 16, generator=g)
    topk = [[3, 1], [0, 2], [1, 1], [2, 3], [0, 3]]
    router = [[0.6, 0.4]] * 5
    ref = omoe.naive_swiglu(x, weights, topk, router)
    got = omoe.grouped_swiglu(x, weights, omoe.plan_groups(topk, 4), router)
    assert float((ref - got).abs().max()) < 1e-5


def test_router_oracles():
    # tests/test_mlx_numerics.py:69-89 restated on the oracle
    torch.manual_seed(2)
    x = torch.randn(3, 16)
    w = torch.randn(8, 16) * 0.1
    b = torch.randn(8)
    scores = omoe.sqrtsoftplus_scores(x, w)
    want = torch.sqrt(torch.nn.functional.softplus(x @ w.T))
    torch.testing.assert_close(scores, want, rtol=1e-6, atol=1e-6)
    wts, idx = omoe.route_topk(scores, b, 2)
    ref_idx = (scores + b).topk(2, dim=-1)[1]
    assert sorted(idx.flatten().tolist()) == sorted(ref_idx.flatten().tolist())
    torch.testing.assert_close(wts.sum(-1), torch.full((3,), 1.5))
    p, i = omoe.route_softmax_topk(torch.randn(4, 256), 8)
    torch.testing.assert_close(p.sum(-1), torch.ones(4))
    assert (i[:, :-1] != i[:, 1:]).all()
