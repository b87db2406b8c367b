"""Device align_block_size (ds_moe_align) vs the reference golden vectors
(tests/test_audit.py:37-67 cases, generated from src/deepseeker/moe_align.py)
and vs the CPU restatement on seeded random inputs; bit-exact."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from deepseeker import moe_align
from oracle import moe as omoe

pytestmark = pytest.mark.gpu


def check(topk, block, E):
    got = moe_align.align_block_size(topk, block, E)
    ref = omoe.align_block_size(topk, block, E)
    np.testing.assert_array_equal(got[0], ref[0])
    np.testing.assert_array_equal(got[1], ref[1])
    assert got[2] == ref[2]
    assert got[0].dtype == np.int64 and got[1].dtype == np.int64


def test_golden_vectors(golden, cuda):
    topk = np.array([[1, 2, 3], [0, 1, 3], [0, 2, 3], [0, 1, 2]])
    s, e, n = moe_align.align_block_size(topk, 4, 4)
    np.testing.assert_array_equal(s, golden["align_doc_sorted"])
    np.testing.assert_array_equal(e, golden["align_doc_experts"])
    assert n == int(golden["align_doc_npad"][0]) == 16
    s, e, n = moe_align.align_block_size(golden["align_rand_topk"], 16, 384)
    np.testing.assert_array_equal(s, golden["align_rand_sorted"])
    np.testing.assert_array_equal(e, golden["align_rand_experts"])
    assert n == int(golden["align_rand_npad"][0])


@pytest.mark.parametrize("M,K,E,block,seed", [
    (1, 1, 1, 1, 0), (3, 2, 5, 1, 1), (7, 3, 4, 4, 2), (256, 6, 384, 16, 3), (100, 8, 256, 64, 4),
    (2048, 8, 256, 16, 5), (16384, 8, 256, 16, 6), (33, 5, 1024, 7, 7), (1000, 1, 3, 128, 8)])
def test_random_vs_oracle(M, K, E, block, seed, cuda):
    rng = np.random.default_rng(seed)
    check(rng.integers(0, E, size=(M, K)), block, E)


def test_skewed_and_single_expert(cuda):
    rng = np.random.default_rng(9)
    p = 1.0 / np.arange(1, 257) ** 1.1
    check(rng.choice(256, size=(4096, 8), p=p / p.sum()), 16, 256)
    check(np.zeros((500, 4), dtype=np.int64), 16, 8)
    check(np.full((31, 1), 7), 32, 8)


def test_empty_and_errors(cuda):
    s, e, n = moe_align.align_block_size(np.zeros((0, 4), dtype=np.int64), 16, 8)
    assert s.size == 0 and e.size == 0 and n == 0
    with pytest.raises(ValueError):
        moe_align.align_block_size(np.array([1, 2, 3]), 4, 4)
    with pytest.raises(ValueError):
        moe_align.align_block_size(np.array([[0, 99]]), 4, 4)
    with pytest.raises(ValueError):
        moe_align.align_block_size(np.array([[0, 1]]), 0, 4)


def test_device_reports_out_of_range(cuda):
    ids = torch.tensor([[0, 5], [1, 2]], dtype=torch.int32, device=cuda)
    _, _, n = moe_align.align_block_size_device(ids, 4, 4)
    assert int(n.item()) == -1
    ids = torch.tensor([[0, -1]], dtype=torch.int32, device=cuda)
    _, _, n = moe_align.align_block_size_device(ids, 4, 4)
    assert int(n.item()) == -1
