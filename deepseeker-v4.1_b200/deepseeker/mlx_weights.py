"""Weight-format helpers -- drop-in for the format half of the reference's ``deepseeker.mlx_weights``.

Reference: src/deepseeker/mlx_weights.py:1-166.  The SSD loaders of that
module (ExpertLoader, DenseLoader, pread pools) are not part of this build:
every expert is resident in HBM.

Device work (FP8 block dequant, FP4 row-major dequant, q3 dequant) runs in
libdeepseeker_b200.so; the rest is host-side format plumbing (tables,
reinterpretation, shape validation) exactly as in the reference.
"""
from __future__ import annotations

import os

import numpy as np
import torch

from . import _abi
from ._dev import ptr, require_cuda, stream_handle, to_device
from .metal_fp4 import FP4_TABLE, _SCALE_TABLE
from .metal_fp4 import dequant as _fp4_dequant

__all__ = ["FP4_TABLE", "E4M3_TABLE", "decode_u8m0", "dequant_fp8_block", "pack_fp4_mxfp4",
           "unpack_int3_affine", "Q3_GROUP_SIZE", "Q3_BITS", "dequant_fp4_rowmajor", "dequant_q3"]


def _build_e4m3() -> np.ndarray:
    """OCP e4m3fn: bias 7, subnormals m/8 * 2^-6, only S.1111.111 is NaN."""
    b = np.arange(256)
    sign = np.where(b & 0x80, -1.0, 1.0)
    e = (b >> 3) & 0xF
    m = (b & 7).astype(np.float64)
    mag = np.where(e == 0, m / 8.0 * 2.0 ** -6, (1.0 + m / 8.0) * np.exp2(e - 7.0))
    t = (sign * mag).astype(np.float32)
    t[(e == 0xF) & ((b & 7) == 7)] = np.nan
    return t


E4M3_TABLE = _build_e4m3()


def _check_e4m3_table() -> None:
    """Cross-check against torch's float8_e4m3fn decode (as the reference does at import)."""
    want = torch.frombuffer(bytearray(range(256)), dtype=torch.float8_e4m3fn).float().numpy()
    same = (np.isnan(want) & np.isnan(E4M3_TABLE)) | (want == E4M3_TABLE)
    if not same.all():
        raise RuntimeError(f"E4M3_TABLE mismatch at bytes {np.where(~same)[0][:8].tolist()}")


_check_e4m3_table()

Q3_GROUP_SIZE = int(os.environ.get("DEEPSEEKER_Q3_GROUP", "64"))
Q3_BITS = int(os.environ.get("DEEPSEEKER_Q3_BITS", "3"))


def decode_u8m0(raw: np.ndarray) -> np.ndarray:
    """ue8m0 bytes -> f32 powers of two (0xFF -> NaN); host-side format helper."""
    raw = np.asarray(raw)
    if raw.dtype == np.uint8:
        return _SCALE_TABLE[raw]
    bits = raw.astype(np.int64)
    out = np.ldexp(np.float64(1.0), bits - 127)
    out[bits == 0xFF] = np.nan
    return out.astype(np.float32)


def dequant_fp8_block(packed: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """[R, C] e4m3 bytes + [R//32, C//32] ue8m0 scales -> f32 (device kernel)."""
    rows, cols = packed.shape
    assert rows % 32 == 0 and cols % 32 == 0, (packed.shape, scales.shape)
    assert scales.shape == (rows // 32, cols // 32), (packed.shape, scales.shape)
    p = to_device(np.ascontiguousarray(packed, dtype=np.uint8))
    s = to_device(np.ascontiguousarray(scales, dtype=np.uint8))
    out = torch.empty((rows, cols), dtype=torch.float32, device=p.device)
    _abi.call("ds_fp8_block_dequant", ptr(p), rows, cols, ptr(s), ptr(out), stream_handle(p.device))
    return out.cpu().numpy()


def pack_fp4_mxfp4(wdata: bytes, sdata: bytes, rows: int, pair_cols: int) -> tuple[np.ndarray, np.ndarray]:
    """On-disk fp4 bytes -> (u32 words [rows, pair_cols/4], u8 scales [rows, pair_cols/16]).

    A little-endian reinterpretation only (8 codes per word, first code in the
    low nibble); the device kernels consume exactly these operands.
    """
    if pair_cols % 4:
        raise ValueError(f"pair_cols {pair_cols} not divisible by 4")
    w = np.frombuffer(wdata, dtype=np.uint8).reshape(rows, pair_cols)
    n_scales = pair_cols // 16
    s = np.frombuffer(sdata, dtype=np.uint8)
    if s.size != rows * n_scales:
        raise ValueError(f"scale bytes {s.size} != {rows * n_scales}")
    return w.view(np.uint32), s.reshape(rows, n_scales)


def unpack_int3_affine(wdata, sdata, bdata, weight_shape, scale_shape) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Stored q3 payload bytes -> (u32 words [rows, words], f16 scales, f16 biases [rows, groups]).

    Validates that the word count matches groups * 64 * 3 bits and that the
    scale and bias shapes agree with each other and with the row count;
    raises ValueError otherwise.
    """
    words = np.frombuffer(wdata, dtype="<u4")
    scales = np.frombuffer(sdata, dtype="<f2").reshape(scale_shape)
    biases = np.frombuffer(bdata, dtype="<f2").reshape(-1)
    rows, word_cols = weight_shape
    want_words = (scales.shape[1] * Q3_GROUP_SIZE * Q3_BITS + 31) // 32
    if biases.size != scales.size or scales.shape[0] != rows or want_words != word_cols:
        raise ValueError(
            f"q3 scale/bias shape mismatch against manifest (weight {weight_shape}, scale {scales.shape})")
    return words.reshape(rows, word_cols), scales, biases.reshape(scales.shape)


def dequant_fp4_rowmajor(packed: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """Flat fp4 pairs (low nibble first) + raw per-32 ue8m0 scales -> f32 (device kernel)."""
    n = packed.size * 2
    n_scales = (n + 31) // 32
    assert scales.size == n_scales, (packed.size, scales.size, n)
    p = to_device(np.frombuffer(np.ascontiguousarray(packed).tobytes(), dtype=np.uint8))
    s = to_device(np.ascontiguousarray(scales, dtype=np.uint8).reshape(-1))
    return _fp4_dequant(p, s, torch.float32).cpu().numpy()


def dequant_q3(words, scales, biases, group_size: int = 64, bits: int = 3,
               out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """q3 payload -> dense [rows, cols] on the device: f32(scale) * q + f32(bias).

    ``words`` [rows, cols*3/32] u32 (or int32 view), ``scales``/``biases``
    [rows, cols/64] f16; numpy arrays are copied to the current device.
    Replaces ``mx.dequantize(..., group_size=64, bits=3)``.
    """
    if group_size != 64 or bits != 3:
        raise NotImplementedError("only group_size=64, bits=3 is implemented")
    if isinstance(words, np.ndarray):
        words = torch.from_numpy(np.ascontiguousarray(words).view(np.int32))
    if isinstance(scales, np.ndarray):
        scales = torch.from_numpy(np.ascontiguousarray(scales, dtype=np.float16))
    if isinstance(biases, np.ndarray):
        biases = torch.from_numpy(np.ascontiguousarray(biases, dtype=np.float16))
    dev = next((t.device for t in (words, scales, biases) if t.is_cuda), torch.device("cuda"))
    words = words.to(dev).contiguous()
    scales = require_cuda(scales.to(dev), "scales", torch.float16)
    biases = require_cuda(biases.to(dev), "biases", torch.float16)
    rows, groups = scales.shape
    if biases.shape != scales.shape:
        raise ValueError(f"biases {tuple(biases.shape)} != scales {tuple(scales.shape)}")
    cols = groups * 64
    if words.numel() != rows * cols * 3 // 32:
        raise ValueError(f"words hold {words.numel()} u32, expected {rows * cols * 3 // 32}")
    out = torch.empty((rows, cols), dtype=out_dtype, device=dev)
    odt = _abi.DS_BF16 if out_dtype == torch.bfloat16 else _abi.DS_F32
    _abi.call("ds_q3_dequant", ptr(words), ptr(scales), ptr(biases), rows, cols, ptr(out), odt,
              stream_handle(dev))
    return out
