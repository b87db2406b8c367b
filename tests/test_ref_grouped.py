"""The reference's tests/test_grouped.py:29-58 run against the drop-in
``deepseeker.grouped``.  The reference draws its tiny weights with MLX's
random generator; these are drawn with torch's, same shapes and scales."""
from __future__ import annotations

import pytest
import torch

from deepseeker.grouped import grouped_swiglu, naive_swiglu, plan_groups


def tiny_weights(device):
    g = torch.Generator().manual_seed(0)
    weights = {}
    for expert in range(4):
        gate = torch.randn(16, 8, generator=g) * 0.1
        up = torch.randn(16, 8, generator=g) * 0.1
        down = torch.randn(8, 16, generator=g) * 0.1
        weights[expert] = (gate.to(device), up.to(device), down.to(device))
    x = torch.randn(5, 16, generator=g).to(device)
    return weights, x


def test_plan_groups_stable_and_complete():
    topk = [[2, 0], [1, 2], [0, 0]]
    groups = plan_groups(topk, 3)
    assert groups == {2: [(0, 0), (1, 1)], 0: [(0, 1), (2, 0), (2, 1)], 1: [(1, 0)]}
    assert plan_groups([[], []], 3) == {}
    try:
        plan_groups([[9]], 3)
    except ValueError:
        pass
    else:
        raise AssertionError("expected ValueError")


@pytest.mark.gpu
def test_grouped_matches_naive(cuda):
    weights, x = tiny_weights(cuda)
    topk = [[3, 1], [0, 2], [1, 1], [2, 3], [0, 3]]
    router = [[0.6, 0.4]] * 5
    groups = plan_groups(topk, 4)
    ref = naive_swiglu(x, weights, topk, router)
    got = grouped_swiglu(x, weights, groups, router)
    diff = float((ref - got).abs().max())
    assert diff < 1e-4


@pytest.mark.gpu
def test_grouped_without_router(cuda):
    weights, x = tiny_weights(cuda)
    topk = [[0, 1], [2, 3]]
    groups = plan_groups(topk, 4)
    ref = naive_swiglu(x, weights, topk)
    got = grouped_swiglu(x, weights, groups)
    diff = float((ref - got).abs().max())
    assert diff < 1e-4
