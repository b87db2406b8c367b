"""FP4 e2m1 dequantisation on B200 -- drop-in for the reference's ``deepseeker.metal_fp4``.

Reference: src/deepseeker/metal_fp4.py.  On-disk layout: two e2m1 codes per
byte, LOW nibble first, decoded through ``FP4_TABLE`` (code 8 is +0.0), one
ue8m0 power-of-two scale per 32 elements (2^(b-127), 0xFF -> NaN).

``metal_dequant`` keeps the reference name and contract (host numpy in, host
f32 out, ValueError on a scale-count mismatch; metal_fp4.py:139-155) but runs
the sm_100a kernel ``ds_fp4_dequant``.  ``dequant`` is the device-resident form
(replaces the bf16/u8-scale Metal path used by the expert loader,
mlx_weights.py:340-360).  ``reference_dequant`` (numpy) and
``torch_reference`` (torch CPU) keep the reference's two host-side
references of the same math (metal_fp4.py:122-131, 158-168), so callers and
tests that cross-check the device result against them work unchanged; the
device kernel is bit-exact with both.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _abi
from ._dev import ptr, require_cuda, stream_handle, to_device

FP4_TABLE = np.array(
    [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
     0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0],
    dtype=np.float32,
)
BLOCK = 32


def _u8m0_table() -> np.ndarray:
    t = np.ldexp(np.float64(1.0), np.arange(256) - 127)
    t[255] = np.nan  # 2^128 is not representable; the format defines 0xFF as NaN
    t = t.astype(np.float32)
    return t


_SCALE_TABLE = _u8m0_table()


def decode_scales_u8m0(raw: bytes) -> np.ndarray:
    """ue8m0 bytes -> f32 powers of two (0xFF -> NaN); host-side format helper."""
    return _SCALE_TABLE[np.frombuffer(raw, dtype=np.uint8)]


def dequant(packed: torch.Tensor, scales: torch.Tensor, out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Device e2m1 dequant: packed u8 [..] (flat), scales f32 or raw u8 (ue8m0), -> 1-D tensor.

    n = 2 * packed.numel(); scales.numel() must be ceil(n / 32).
    """
    packed = require_cuda(packed, "packed", torch.uint8)
    scales = require_cuda(scales, "scales", (torch.float32, torch.uint8))
    n = packed.numel() * 2
    if scales.numel() != (n + BLOCK - 1) // BLOCK:
        raise ValueError("scales must cover ceil(n/32) blocks")
    if out_dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("out_dtype must be torch.float32 or torch.bfloat16")
    out = torch.empty(n, dtype=out_dtype, device=packed.device)
    kind = _abi.DS_U8 if scales.dtype == torch.uint8 else _abi.DS_F32
    odt = _abi.DS_BF16 if out_dtype == torch.bfloat16 else _abi.DS_F32
    with torch.cuda.device(packed.device):
        _abi.call("ds_fp4_dequant", ptr(packed), packed.numel(), ptr(scales), kind, scales.numel(),
                  ptr(out), odt, stream_handle(packed.device))
    return out


def metal_dequant(packed: np.ndarray, scales_f32: np.ndarray) -> np.ndarray:
    """Device e2m1 dequant of host arrays; returns a float32 host array, exact vs reference."""
    n = packed.size * 2
    if scales_f32.size != (n + BLOCK - 1) // BLOCK:
        raise ValueError("scales must cover ceil(n/32) blocks")
    p = to_device(np.frombuffer(np.ascontiguousarray(packed).tobytes(), dtype=np.uint8))
    s = to_device(np.ascontiguousarray(scales_f32, dtype=np.float32).reshape(-1))
    out = dequant(p, s, torch.float32)
    return out.cpu().numpy()


def reference_dequant(packed: np.ndarray, scales_f32: np.ndarray) -> np.ndarray:
    """Host numpy form of the dequant (metal_fp4.py:122-131): FP4_TABLE[nibble]
    (low nibble = even element) times the block's f32 scale, one f32 multiply
    per element; ``scales_f32`` must hold n/32 entries."""
    raw = np.frombuffer(np.ascontiguousarray(packed).tobytes(), dtype=np.uint8)
    vals = np.empty(raw.size * 2, dtype=np.float32)
    vals[0::2] = FP4_TABLE[raw & 0x0F]
    vals[1::2] = FP4_TABLE[raw >> 4]
    return vals * np.repeat(np.asarray(scales_f32, dtype=np.float32).reshape(-1), BLOCK)


def torch_reference(packed: np.ndarray, scales_f32: np.ndarray) -> torch.Tensor:
    """Host torch form of the same dequant (metal_fp4.py:158-168), an
    independent cross-check of ``reference_dequant``; returns a CPU tensor."""
    table = torch.from_numpy(FP4_TABLE.copy())
    raw = torch.frombuffer(bytearray(np.ascontiguousarray(packed).tobytes()), dtype=torch.uint8)
    vals = torch.empty(raw.numel() * 2, dtype=torch.float32)
    vals[0::2] = table[(raw & 0x0F).long()]
    vals[1::2] = table[(raw >> 4).long()]
    rep = torch.from_numpy(np.ascontiguousarray(scales_f32, dtype=np.float32).reshape(-1)).repeat_interleave(BLOCK)
    return vals * rep
