"""Grouped planner and Zipf router: host logic, no GPU (grouped.py:19-31 golden)."""
from __future__ import annotations

import json

import pytest
import torch

from deepseeker import grouped, synthetic


def test_plan_groups_matches_reference_golden(golden):
    groups = grouped.plan_groups([[2, 0], [1, 2], [0, 0]], 3)
    assert groups == {2: [(0, 0), (1, 1)], 0: [(0, 1), (2, 0), (2, 1)], 1: [(1, 0)]}
    assert json.dumps({str(k): v for k, v in groups.items()}) == golden["_hashes"]["plan_groups_golden"]
    assert grouped.plan_groups([[], []], 3) == {}
    with pytest.raises(ValueError):
        grouped.plan_groups([[9]], 3)


def test_zipf_routing_shape_distinct_and_skewed():
    ids, w = synthetic.zipf_routing(2048, 256, 8, s=1.1, seed=3, device="cpu")
    assert ids.shape == (2048, 8) and w.shape == (2048, 8)
    assert ids.dtype == torch.int32 and w.dtype == torch.float32
    assert int(ids.min()) >= 0 and int(ids.max()) < 256
    srt = ids.sort(dim=1).values
    assert bool((srt[:, 1:] != srt[:, :-1]).all()), "experts of a token must be distinct"
    torch.testing.assert_close(w.sum(1), torch.ones(2048))
    counts = torch.bincount(ids.flatten().long(), minlength=256).sort(descending=True).values
    assert int(counts[0]) > 1000 and int(counts[-1]) < 64   # heavy head, light tail
    ids2, _ = synthetic.zipf_routing(2048, 256, 8, s=1.1, seed=3, device="cpu")
    assert torch.equal(ids, ids2)
