"""The reference's tests/test_metal_fp4.py (the parts that need no model
checkpoint: lines 35-53 and 98-101), run against the drop-in
``deepseeker.metal_fp4``; only the import path differs."""
from __future__ import annotations

import numpy as np
import pytest

from deepseeker.metal_fp4 import FP4_TABLE, decode_scales_u8m0, metal_dequant, reference_dequant, torch_reference


def test_table_spot_values():
    assert FP4_TABLE[0x7] == 6.0
    assert FP4_TABLE[0xF] == -6.0
    assert FP4_TABLE[0x8] == 0.0
    assert decode_scales_u8m0(bytes([127]))[0] == 1.0
    assert decode_scales_u8m0(bytes([128]))[0] == 2.0
    assert np.isnan(decode_scales_u8m0(bytes([0xFF]))[0])


def test_host_references_agree():
    rng = np.random.default_rng(3)
    packed = rng.integers(0, 256, size=512, dtype=np.uint8)
    scales = np.exp2(rng.integers(-3, 3, size=32).astype(np.float32))
    np.testing.assert_array_equal(reference_dequant(packed, scales), torch_reference(packed, scales).numpy())


@pytest.mark.gpu
def test_metal_matches_references_random(cuda):
    rng = np.random.default_rng(3)
    packed = rng.integers(0, 256, size=512, dtype=np.uint8)  # 1024 elems
    scales = np.exp2(rng.integers(-3, 3, size=32).astype(np.float32))
    ref = reference_dequant(packed, scales)
    got = metal_dequant(packed, scales)
    assert got.shape == (1024,)
    np.testing.assert_array_equal(got, ref)
    torch_vals = torch_reference(packed, scales).numpy()
    np.testing.assert_array_equal(got, torch_vals)


def test_bad_scales_rejected():
    packed = np.zeros(128, dtype=np.uint8)
    with pytest.raises(ValueError):
        metal_dequant(packed, np.ones(3, dtype=np.float32))
