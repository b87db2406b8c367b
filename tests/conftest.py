"""Shared test setup: import paths, the `gpu` marker, golden vectors, seeded bank builders."""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "deepseeker-v4.1_b200"
for p in (str(PKG), str(ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    with np.load(GOLDEN / "ref_vectors.npz") as z:
        vec = {k: z[k] for k in z.files}
    vec["_hashes"] = json.loads((GOLDEN / "ref_hashes.json").read_text())
    return vec


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)
