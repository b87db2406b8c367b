"""ctypes binding of libdeepseeker_b200.so (the C ABI declared in include/deepseeker_b200.h).

The library is the only compute path: if it is missing or cannot be loaded,
every operator raises -- there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, Structure, c_char_p, c_float, c_int, c_int32, c_int64, c_size_t, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libdeepseeker_b200.so"

# status codes
DS_OK, DS_EINVAL, DS_EALIGN, DS_ERANGE, DS_ECUDA, DS_ETIMEOUT, DS_ENOTSUP = range(7)
# element types
DS_F32, DS_BF16, DS_F16, DS_U8 = range(4)
# weight formats
DS_FMT_FP4, DS_FMT_Q3, DS_FMT_BF16 = range(3)
# routing kinds
DS_ROUTE_SOFTMAX, DS_ROUTE_SQRTSOFTPLUS, DS_ROUTE_SCORES = 0, 1, 2


class DsExpertBank(Structure):
    _fields_ = [("format", c_int32), ("n_experts", c_int32), ("rows", c_int32), ("cols", c_int32),
                ("data", c_void_p), ("scales", c_void_p), ("biases", c_void_p), ("scales_tc", c_void_p)]


class DsMoeDesc(Structure):
    _fields_ = [("hidden", c_int32), ("inter", c_int32), ("n_experts", c_int32), ("top_k", c_int32),
                ("w1", DsExpertBank), ("w3", DsExpertBank), ("w2", DsExpertBank),
                ("shared_w1", c_void_p), ("shared_w3", c_void_p), ("shared_w2", c_void_p),
                ("shared_inter", c_int32), ("swiglu_limit", c_float), ("route_before_down", c_int32),
                ("out_f32", c_int32)]


# name -> (restype, argtypes); every symbol include/deepseeker_b200.h declares
SIGNATURES: dict[str, tuple] = {
    "ds_last_error_string": (c_char_p, []),
    "ds_version": (c_int, []),
    "ds_fp4_dequant": (c_int, [c_void_p, c_int64, c_void_p, c_int, c_int64, c_void_p, c_int, c_void_p]),
    "ds_fp8_block_dequant": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p]),
    "ds_q3_dequant": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_int, c_void_p]),
    "ds_q3_quantize": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p]),
    "ds_fp4_quantize": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p]),
    "ds_route_topk": (c_int, [c_void_p, c_void_p, c_int64, c_int, c_int, c_int, c_float, c_void_p,
                              c_void_p, c_void_p]),
    "ds_moe_decode_workspace_size": (c_int, [POINTER(DsMoeDesc), c_int64, POINTER(c_size_t)]),
    "ds_moe_decode": (c_int, [POINTER(DsMoeDesc), c_void_p, c_int, c_int64, c_void_p, c_void_p, c_void_p,
                              c_void_p, c_size_t, c_void_p]),
    "ds_moe_decode_route": (c_int, [POINTER(DsMoeDesc), c_void_p, c_int, c_int64, c_void_p, c_void_p, c_int,
                                    c_float, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "ds_qmm": (c_int, [POINTER(DsExpertBank), c_void_p, c_int, c_int64, c_void_p, c_void_p]),
    "ds_host_device_pointer": (c_int, [c_void_p, POINTER(c_void_p)]),
    "ds_copy_ranges": (c_int, [c_int, POINTER(c_void_p), POINTER(c_void_p), POINTER(c_size_t), c_void_p]),
    "ds_moe_align_capacity": (c_int, [c_int64, c_int, c_int, c_int, POINTER(c_int64), POINTER(c_int64)]),
    "ds_moe_align": (c_int, [c_void_p, c_int64, c_int, c_int, c_int, c_void_p, c_int64, c_void_p, c_int64,
                             c_void_p, c_void_p]),
    "ds_fp4_scale_atoms": (c_int, [c_void_p, c_int64, c_int, c_int, c_void_p, c_void_p]),
    "ds_grouped_scales_size": (c_int, [POINTER(DsMoeDesc), POINTER(c_size_t), POINTER(c_size_t)]),
    "ds_grouped_prepare_scales": (c_int, [POINTER(DsMoeDesc), c_void_p, c_void_p, c_void_p]),
    "ds_grouped_ffn_workspace_size": (c_int, [POINTER(DsMoeDesc), c_int64, POINTER(c_size_t)]),
    "ds_grouped_ffn": (c_int, [POINTER(DsMoeDesc), c_void_p, c_void_p, c_void_p, c_int, c_int64, c_void_p,
                               c_void_p, c_void_p, c_int, c_void_p, c_size_t, c_void_p]),
    "ds_grouped_ffn_fp4_workspace_size": (c_int, [POINTER(DsMoeDesc), c_int64, POINTER(c_size_t)]),
    "ds_grouped_ffn_fp4": (c_int, [POINTER(DsMoeDesc), c_void_p, c_int, c_int64, c_void_p, c_void_p, c_void_p,
                                   c_int, c_void_p, c_size_t, c_void_p]),
    "ds_dense_swiglu_workspace_size": (c_int, [c_int64, c_int, POINTER(c_size_t)]),
    "ds_dense_swiglu": (c_int, [c_void_p, c_int64, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_int64,
                                c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_void_p, c_void_p, c_size_t,
                                c_void_p]),
    "ds_moe_decode_noalloc_max_scratch": (c_size_t, []),
    "ds_moe_decode_noalloc": (c_int, [POINTER(DsMoeDesc), c_void_p, c_int, c_int64, c_void_p, c_void_p,
                                      c_void_p, c_void_p]),
    "ds_moe_decode_noalloc_status": (c_int, [c_void_p, c_void_p]),
    "ds_ep_create": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, POINTER(c_void_p)]),
    "ds_ep_region_bytes": (c_size_t, [c_int, c_int, c_int, c_int]),
    "ds_ep_ipc_handle": (c_int, [c_void_p, c_void_p]),
    "ds_ep_connect": (c_int, [c_void_p, c_void_p]),
    "ds_ep_connect_peers": (c_int, [c_void_p, c_void_p]),
    "ds_ep_decode_workspace_size": (c_int, [c_void_p, POINTER(DsMoeDesc), c_int64, POINTER(c_size_t)]),
    "ds_ep_decode": (c_int, [c_void_p, POINTER(DsMoeDesc), c_int32, c_void_p, c_int64, c_void_p, c_void_p,
                             c_void_p, c_void_p, c_size_t, c_void_p]),
    "ds_ep_status": (c_int, [c_void_p, POINTER(c_int32)]),
    "ds_ep_destroy": (c_int, [c_void_p]),
}

_lib: ctypes.CDLL | None = None


class DsError(RuntimeError):
    """A CUDA-side failure reported by the library (DS_ECUDA, DS_ETIMEOUT...)."""


def lib() -> ctypes.CDLL:
    """Load the library once; raise if it is absent (no fallback)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'`"
                " (the CUDA library is the only implementation of these operators)")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(status: int, what: str) -> None:
    """Map a status code to the reference's exception types."""
    if status == DS_OK:
        return
    msg = lib().ds_last_error_string().decode(errors="replace")
    if status in (DS_EINVAL, DS_EALIGN, DS_ERANGE):
        raise ValueError(f"{what}: {msg}")
    if status == DS_ENOTSUP:
        raise NotImplementedError(f"{what}: {msg}")
    raise DsError(f"{what}: status {status}: {msg}")


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)
