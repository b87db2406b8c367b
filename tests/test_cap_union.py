"""cap_union (host logic of mlx_forward.py:213-254), with the reference's
own cases from tests/test_batch.py:203-249."""
from __future__ import annotations

import numpy as np

from deepseeker.moe import cap_union


def test_cap_union_is_exact_when_the_union_fits():
    idx = np.array([[1, 2, 3], [3, 4, 5]], dtype=np.int64)
    w = np.array([[0.7, 0.5, 0.3], [0.6, 0.5, 0.4]], dtype=np.float32)
    out_i, out_w, coverage = cap_union(idx, w, 8, 5)
    np.testing.assert_array_equal(out_i, idx)
    np.testing.assert_allclose(out_w, w, rtol=1e-6)
    assert coverage == 1.0


def test_cap_union_shrinks_union_and_preserves_each_row_weight_sum():
    rng = np.random.default_rng(0)
    idx = np.array([[0, 1, 2], [0, 3, 4], [0, 5, 6], [1, 3, 5], [2, 4, 6], [7, 8, 9]], dtype=np.int64)
    w = rng.random((6, 3)).astype(np.float32)
    w /= w.sum(axis=1, keepdims=True)
    w *= 1.5
    out_i, out_w, coverage = cap_union(idx, w, 12, 4)
    live = out_i[out_i >= 0]
    assert np.unique(live).size <= 4 + idx.shape[0]
    np.testing.assert_allclose(out_w.sum(axis=1), w.sum(axis=1), rtol=1e-5)
    kept = out_i >= 0
    for r in range(idx.shape[0]):
        vals = out_w[r][kept[r]] / w[r][kept[r]]
        np.testing.assert_allclose(vals, vals[0], rtol=1e-5)
        assert vals[0] >= 1.0 - 1e-6
    assert 0.0 < coverage <= 1.0


def test_cap_union_row_never_loses_every_expert():
    idx = np.array([[90, 91, 92], [1, 2, 3], [1, 2, 4]], dtype=np.int64)
    w = np.array([[0.5, 0.5, 0.5], [5.0, 4.0, 3.0], [5.0, 4.0, 3.0]], dtype=np.float32)
    out_i, out_w, coverage = cap_union(idx, w, 93, 3)
    assert (out_i[0] >= 0).sum() == 1
    np.testing.assert_allclose(out_w[0].sum(), w[0].sum(), rtol=1e-5)
    assert coverage < 1.0


def test_cap_union_strict_keeps_exactly_the_budget():
    idx = np.array([[90, 91, 92], [1, 2, 3], [1, 2, 4]], dtype=np.int64)
    w = np.array([[0.5, 0.5, 0.5], [5.0, 4.0, 3.0], [5.0, 4.0, 3.0]], dtype=np.float32)
    out_i, _, _ = cap_union(idx, w, 93, 3, strict=True)
    assert np.unique(out_i[out_i >= 0]).size == 3
    assert (out_i[0] < 0).all()
