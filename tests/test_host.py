"""Host-side logic of the drop-in modules (no GPU): shape contracts, variant
selection, format reinterpretation, argument validation before any launch."""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from deepseeker import metal_fp4, mlx_weights as W, requant, variant_q3
from oracle import fp4 as ofp4


def test_tables_match_oracle():
    np.testing.assert_array_equal(metal_fp4.FP4_TABLE, ofp4.FP4_TABLE)
    assert metal_fp4.BLOCK == 32
    a = metal_fp4.decode_scales_u8m0(bytes(range(256)))
    b = ofp4.decode_scales_u8m0(bytes(range(256)))
    assert ((a.view(np.uint32) == b.view(np.uint32)) | (np.isnan(a) & np.isnan(b))).all()
    # tests/test_metal_fp4.py:35-41
    assert metal_fp4.decode_scales_u8m0(bytes([127]))[0] == 1.0
    assert metal_fp4.decode_scales_u8m0(bytes([128]))[0] == 2.0
    assert np.isnan(metal_fp4.decode_scales_u8m0(bytes([0xFF]))[0])
    c = W.decode_u8m0(np.arange(256, dtype=np.uint8))
    assert ((c.view(np.uint32) == b.view(np.uint32)) | (np.isnan(c) & np.isnan(b))).all()
    d = W.decode_u8m0(np.arange(256, dtype=np.int32))
    assert ((d.view(np.uint32) == b.view(np.uint32)) | (np.isnan(d) & np.isnan(b))).all()


def test_e4m3_table_spots():
    # tests/test_mlx_weights.py:47-61
    T = W.E4M3_TABLE
    assert T[0x00] == 0.0 and T[0x40] == 2.0 and T[0x3C] == 1.5 and T[0xC0] == -2.0
    assert T[0x78] == 256.0 and T[0x7E] == 448.0
    assert np.isnan(T[0x7F]) and np.isnan(T[0xFF])
    want = torch.frombuffer(bytearray(range(256)), dtype=torch.float8_e4m3fn).float().numpy()
    assert ((np.isnan(want) & np.isnan(T)) | (want == T)).all()


def test_bad_scales_rejected_before_launch():
    # tests/test_metal_fp4.py:98-101: ValueError, no device needed
    with pytest.raises(ValueError):
        metal_fp4.metal_dequant(np.zeros(128, dtype=np.uint8), np.ones(3, dtype=np.float32))


def test_parse_layers_and_experts():
    # tests/test_q3.py:38-46
    assert requant.parse_layers("20-23") == [20, 21, 22, 23]
    assert requant.parse_layers("2,5,7") == [2, 5, 7]
    assert requant.parse_layers("0,6-8") == [0, 6, 7, 8]
    assert requant.parse_experts(None) == list(range(384))
    assert requant.parse_experts("3-5") == [3, 4, 5]
    assert requant.FP4_EXPERT_BYTES == 18800640


def test_is_q3_variant_names():
    assert variant_q3.is_q3("1017-Q3") and variant_q3.is_q3("q3") and variant_q3.is_q3("1017-q3")
    assert not variant_q3.is_q3("1017") and not variant_q3.is_q3("")
    old = os.environ.pop("DEEPSEEKER_VARIANT", None)
    try:
        assert not variant_q3.is_q3(None)
        os.environ["DEEPSEEKER_VARIANT"] = "x-Q3"
        assert variant_q3.is_q3(None)
    finally:
        os.environ.pop("DEEPSEEKER_VARIANT", None)
        if old is not None:
            os.environ["DEEPSEEKER_VARIANT"] = old


def test_paths_for_variant(tmp_path, monkeypatch):
    # tests/test_q3.py:49-77
    rev = "abc123"
    profile = tmp_path / "profiles" / "deepseek-v4.1-flash" / rev
    profile.mkdir(parents=True)
    (tmp_path / "models" / "DeepSeek-V4.1-Flash-Q3").mkdir(parents=True)
    monkeypatch.delenv("DEEPSEEKER_Q3_MANIFEST", raising=False)
    root, man = variant_q3.paths_for_variant(rev, tmp_path, "DeepSeek-V4.1-Flash")
    assert man == profile / "model-manifest.json"
    assert root == tmp_path / "models" / "DeepSeek-V4.1-Flash-1017"
    root, man = variant_q3.paths_for_variant(rev, tmp_path, "DeepSeek-V4.1-Flash", variant="1017-Q3")
    assert man == profile / "model-manifest-q3.json"
    assert root == tmp_path / "models" / "DeepSeek-V4.1-Flash-Q3"
    monkeypatch.setenv("DEEPSEEKER_Q3_MANIFEST", "model-manifest-qprobe.json")
    _, man = variant_q3.paths_for_variant(rev, tmp_path, "DeepSeek-V4.1-Flash", variant="q3")
    assert man == profile / "model-manifest-qprobe.json"


def test_unpack_int3_affine_contract():
    # tests/test_q3.py:108-129
    words = np.zeros((4, 24), dtype="<u4").tobytes()
    scales = np.zeros((4, 4), dtype="<f2").tobytes()
    with pytest.raises(ValueError):
        W.unpack_int3_affine(words, scales, np.zeros((4, 5), dtype="<f2").tobytes(), (4, 24), (4, 4))
    with pytest.raises(ValueError):
        W.unpack_int3_affine(words, np.zeros((3, 4), dtype="<f2").tobytes(),
                             np.zeros((4, 4), dtype="<f2").tobytes(), (4, 24), (4, 4))
    rows, cols = 2, 128
    wr = (cols * 3 + 31) // 32
    w, s, b = W.unpack_int3_affine(np.zeros((rows, wr), "<u4").tobytes(), np.full((rows, 2), 120, "<f2").tobytes(),
                                   np.zeros((rows, 2), "<f2").tobytes(), (rows, wr), (rows, 2))
    assert w.shape == (rows, wr) and s.shape == (rows, 2) and b.shape == (rows, 2)
    assert W.Q3_GROUP_SIZE == 64 and W.Q3_BITS == 3


def test_pack_fp4_mxfp4_is_a_view():
    rng = np.random.default_rng(5)
    raw = rng.integers(0, 256, size=(4, 32), dtype=np.uint8)
    sc = rng.integers(120, 135, size=(4, 2), dtype=np.uint8)
    w, s = W.pack_fp4_mxfp4(raw.tobytes(), sc.tobytes(), 4, 32)
    assert w.dtype == np.uint32 and w.shape == (4, 8) and s.shape == (4, 2)
    np.testing.assert_array_equal(w.view(np.uint8), raw)
    with pytest.raises(ValueError):
        W.pack_fp4_mxfp4(raw.tobytes(), sc.tobytes(), 4, 30)
    with pytest.raises(ValueError):
        W.pack_fp4_mxfp4(raw.tobytes(), sc.tobytes()[:-1], 4, 32)


def test_q3_geometry_arguments():
    with pytest.raises(NotImplementedError):
        W.dequant_q3(np.zeros((1, 6), np.uint32), np.zeros((1, 1), np.float16), np.zeros((1, 1), np.float16),
                     group_size=32)
    with pytest.raises(NotImplementedError):
        requant.convert_tensor(np.zeros(256, np.float32), 1, 256, bits=4)
