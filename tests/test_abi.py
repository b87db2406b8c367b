"""The C-ABI library builds for sm_100a, loads without a GPU and exports every
symbol include/deepseeker_b200.h declares (no compute call is made here)."""
from __future__ import annotations

import re
from pathlib import Path

import pytest

from deepseeker import _abi, _build

HEADER = Path(__file__).resolve().parents[1] / "include" / "deepseeker_b200.h"


def declared_symbols() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(ds_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    _build.build(verbose=False)
    return _abi.lib()


def test_header_and_binding_agree():
    syms = declared_symbols()
    assert len(syms) >= 10
    assert set(syms) == set(_abi.SIGNATURES), set(syms) ^ set(_abi.SIGNATURES)


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert lib.ds_version() >= 100
    assert lib.ds_last_error_string() == b""


def test_host_side_validation_needs_no_gpu(lib):
    # invalid arguments are rejected before any CUDA call, with a message
    st = lib.ds_fp4_dequant(None, 64, None, _abi.DS_U8, 3, None, _abi.DS_F32, None)
    assert st == _abi.DS_EINVAL
    assert b"ceil(n/32)" in lib.ds_last_error_string()
    st = lib.ds_q3_dequant(None, None, None, 4, 100, None, _abi.DS_F32, None)
    assert st == _abi.DS_EINVAL
    with pytest.raises(ValueError):
        _abi.check(st, "ds_q3_dequant")
    st = lib.ds_route_topk(None, None, 1, 2048, 8, 0, 1.0, None, None, None)
    assert st == _abi.DS_EINVAL


def test_no_fast_math_in_build_flags():
    flags = " ".join(_build.CFLAGS + _build.ARCH)
    assert "fast_math" not in flags and "ftz=true" not in flags
    assert "arch=compute_100a,code=sm_100a" in flags
