"""Device dequant / quantise kernels are bit-exact with the pinned oracle
(NaN-aware; +0.0 for code 8; subnormal and NaN scale bytes included)."""
from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

from deepseeker import metal_fp4, mlx_weights as W, requant, synthetic
from oracle import fp4 as ofp4
from oracle import q3 as oq3

pytestmark = pytest.mark.gpu


def bits_equal(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    assert a.shape == b.shape, (a.shape, b.shape)
    same = (a.view(np.uint32) == b.view(np.uint32)) | (np.isnan(a) & np.isnan(b))
    assert same.all(), (np.where(~same)[0][:8], a[~same][:8], b[~same][:8])


def test_metal_matches_references_random(golden, cuda):
    # tests/test_metal_fp4.py:44-53
    got = metal_fp4.metal_dequant(golden["fp4_seed3_packed"], golden["fp4_seed3_scales"])
    assert got.shape == (1024,)
    bits_equal(got, golden["fp4_seed3_out"])
    bits_equal(got, golden["fp4_seed3_torch"])


def test_rowmajor_matches_reference(golden, cuda):
    # tests/test_mlx_weights.py:77-88 and tests/test_q3.py:132-141
    bits_equal(W.dequant_fp4_rowmajor(golden["fp4_seed2_packed"], golden["fp4_seed2_raw_scales"]),
               golden["fp4_seed2_out"])
    bits_equal(W.dequant_fp4_rowmajor(np.array([0x13], np.uint8), np.array([128], np.uint8)),
               golden["fp4_nibble_out"])
    bits_equal(W.dequant_fp4_rowmajor(np.array([0x21, 0x9F, 0x78], np.uint8), np.array([130], np.uint8)),
               golden["fp4_tail_out"])


def test_exhaustive_every_byte_every_scale(golden, cuda):
    packed = np.tile(np.arange(256, dtype=np.uint8), 256)
    scales = np.repeat(np.arange(256, dtype=np.uint8), 16)
    got = W.dequant_fp4_rowmajor(packed, scales)
    bits_equal(got, golden["fp4_exhaustive_out"])
    # +0.0 (not -0.0) for code 8 under every finite scale byte (0..254)
    per_scale = got.reshape(256, 256, 2)            # [scale byte, packed byte, nibble]
    lo_is_8 = (np.arange(256) & 0xF) == 8
    assert not np.signbit(per_scale[:255, lo_is_8, 0]).any()
    hi_is_8 = (np.arange(256) >> 4) == 8
    assert not np.signbit(per_scale[:255, hi_is_8, 1]).any()
    # bf16 output == RNE of the f32 reference
    dev = torch.device("cuda")
    out = metal_fp4.dequant(torch.from_numpy(packed).to(dev), torch.from_numpy(scales).to(dev), torch.bfloat16)
    want = torch.from_numpy(golden["fp4_exhaustive_out"]).to(torch.bfloat16)
    g = out.cpu()
    same = (g.view(torch.int16) == want.view(torch.int16)) | (torch.isnan(g) & torch.isnan(want))
    assert bool(same.all())


def test_bench_fp4_seed9_hash(golden, cuda):
    # scripts/bench_fp4.py:49-58: maxdiff must be exactly 0 on 5120 x 2304
    rng = np.random.default_rng(9)
    packed = rng.integers(0, 256, size=(5120 * 2304) // 2, dtype=np.uint8)
    scales = np.exp2(rng.integers(-2, 3, size=(5120 * 2304) // 32).astype(np.float32))
    got = metal_fp4.metal_dequant(packed, scales)
    assert hashlib.sha256(got.tobytes()).hexdigest() == golden["_hashes"]["bench_fp4_seed9_out"]


def test_unaligned_and_tail_paths(cuda):
    rng = np.random.default_rng(11)
    buf = rng.integers(0, 256, size=4096 + 17, dtype=np.uint8)
    dev = torch.device("cuda")
    t = torch.from_numpy(buf).to(dev)
    for off, nb in ((1, 4096), (0, 4096 + 17), (3, 999), (0, 1)):
        packed = t[off:off + nb]
        n = 2 * nb
        sc = torch.from_numpy(rng.integers(100, 150, size=(n + 31) // 32, dtype=np.uint8)).to(dev)
        got = metal_fp4.dequant(packed, sc).cpu().numpy()
        bits_equal(got, ofp4.dequant_u8_scales(buf[off:off + nb], sc.cpu().numpy()))


def test_bad_scale_count_rejected(cuda):
    with pytest.raises(ValueError):
        metal_fp4.metal_dequant(np.zeros(128, dtype=np.uint8), np.ones(3, dtype=np.float32))


def test_fp8_block(golden, cuda):
    bits_equal(W.dequant_fp8_block(golden["fp8_seed1_packed"], golden["fp8_seed1_scales"]),
               golden["fp8_seed1_out"])
    rng = np.random.default_rng(4)
    p = rng.integers(0, 256, size=(64, 96), dtype=np.uint8)
    s = rng.integers(0, 256, size=(2, 3), dtype=np.uint8)
    with np.errstate(over="ignore", invalid="ignore"):
        bits_equal(W.dequant_fp8_block(p, s), ofp4.dequant_fp8_block(p, s))


def test_fp4_quantizer_matches_oracle(cuda):
    g = torch.Generator().manual_seed(1)
    w = torch.randn(64, 512, generator=g) * 0.02
    w[0, :32] = 0.0                                  # all-zero block
    w[1, :32] = torch.tensor([6.0, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0] * 4)  # exact ties
    w[2, :32] *= 1e30                                 # large exponent
    w[3, :32] *= 1e-30                                # tiny exponent
    p, s = synthetic.quantize_fp4(w.cuda())
    pr, sr = ofp4.quantize_fp4(w.numpy())
    np.testing.assert_array_equal(p.cpu().numpy(), pr)
    np.testing.assert_array_equal(s.cpu().numpy(), sr)


def test_q3_quantize_dequant_match_oracle(cuda):
    g = torch.Generator().manual_seed(7)
    w = torch.randn(16, 320, generator=g) * 0.05
    w[0, :64] = 0.125                                  # constant group: scale 0
    w[1, 64:128] = torch.linspace(-1, 1, 64)
    words, s, b = requant.quantize_q3(w.cuda())
    wr, sr, br = oq3.quantize(w.numpy())
    np.testing.assert_array_equal(words.cpu().numpy().view(np.uint32), wr)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint16), sr.view(np.uint16))
    np.testing.assert_array_equal(b.cpu().numpy().view(np.uint16), br.view(np.uint16))
    got = W.dequant_q3(words, s, b)
    bits_equal(got.cpu().numpy(), oq3.dequant(wr, sr, br))
    got16 = W.dequant_q3(words, s, b, out_dtype=torch.bfloat16).cpu()
    assert bool((got16 == torch.from_numpy(oq3.dequant(wr, sr, br)).to(torch.bfloat16)).all())


def test_convert_tensor_roundtrip_and_geometry(cuda):
    # tests/test_q3.py:89-105 (decode through this build's dequant instead of MLX's)
    rng = np.random.default_rng(7)
    vals = (rng.standard_normal(8 * 256) * 0.05).astype(np.float32)
    words, sraw, braw, rms = requant.convert_tensor(vals, 8, 256, bits=3)
    assert len(words) == 8 * 24 * 4 and len(sraw) == 8 * 4 * 2 and len(braw) == 8 * 4 * 2
    assert 0.0 < rms < 0.08
    wq, sq, bq = W.unpack_int3_affine(words, sraw, braw, (8, 24), (8, 4))
    rt = W.dequant_q3(wq, sq, bq).cpu().numpy().astype(np.float64)
    err = vals.reshape(8, 256).astype(np.float64) - rt
    rms2 = float(np.sqrt(np.mean(err ** 2)) / max(float(np.abs(rt).max()), 1e-9))
    assert abs(rms - rms2) < 1e-6
    wr, sr, br = oq3.quantize(vals.reshape(8, 256))
    assert words == wr.astype("<u4").tobytes() and sraw == sr.astype("<f2").tobytes()
