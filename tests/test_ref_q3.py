"""The reference's tests/test_q3.py:108-141 (shape contracts of the q3
payload and the FP4 row-major interleave), run against the drop-in
``deepseeker.mlx_weights``; only the import path differs."""
from __future__ import annotations

import numpy as np
import pytest

from deepseeker import mlx_weights as W


def test_unpack_int3_affine_rejects_shape_mismatch():
    words = np.zeros((4, 24), dtype="<u4").tobytes()
    scales = np.zeros((4, 4), dtype="<f2").tobytes()
    biases = np.zeros((4, 5), dtype="<f2").tobytes()
    with pytest.raises(ValueError):
        W.unpack_int3_affine(words, scales, biases, (4, 24), (4, 4))
    biases = np.zeros((4, 4), dtype="<f2").tobytes()
    scales_bad = np.zeros((3, 4), dtype="<f2").tobytes()
    with pytest.raises(ValueError):
        W.unpack_int3_affine(words, scales_bad, biases, (4, 24), (4, 4))


def test_unpack_int3_affine_passes_shape_check():
    rows, cols, gs, bits = 2, 128, 64, 3
    words_row = (cols * bits + 31) // 32
    groups = cols // gs
    words = np.zeros((rows, words_row), dtype="<u4").tobytes()
    scales = np.full((rows, groups), 120, dtype="<f2").tobytes()
    biases = np.zeros((rows, groups), dtype="<f2").tobytes()
    w, s, b = W.unpack_int3_affine(words, scales, biases, (rows, words_row), (rows, groups))
    assert w.shape == (rows, words_row)
    assert s.shape == (rows, groups) and b.shape == (rows, groups)


@pytest.mark.gpu
def test_dequant_fp4_rowmajor_interleaving_and_scale(cuda):
    # Two bytes -> four nibble slots, low nibble first.
    # fp4 table index 3 == 1.0 (E2M1), index 1 == 0.5.
    raw = np.array([0x13], dtype=np.uint8)  # low=3, high=1
    gain = W.decode_u8m0(np.array([128], dtype=np.uint8))  # 2.0
    vals = W.dequant_fp4_rowmajor(raw, np.array([128], dtype=np.uint8))
    expect = np.array([W.FP4_TABLE[3], W.FP4_TABLE[1]], dtype=np.float32)
    assert float(gain[0]) == 2.0
    np.testing.assert_allclose(vals, expect * 2.0, rtol=0, atol=0)
