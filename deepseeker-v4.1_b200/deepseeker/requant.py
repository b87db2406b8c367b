"""q3 payload conversion API -- drop-in for the callable part of the reference's
``scripts/requant_experts_3bit.py`` (``parse_layers``, ``parse_experts``,
``convert_tensor``; reference lines 52-83).

``convert_tensor`` quantises on the device with the builder's 3-bit affine
rule (group 64: per-group min/max, scale = (max-min)/7 and bias = min rounded
to f16, q = clamp(rint((w - bias)/scale), 0, 7)), dequantises the result on
the device and reports the same relative-RMS quality figure as the reference
(rms(err) / max|roundtrip|, float64).  The resulting words use this build's
documented 3-bit layout (the reference's MLX packing is MLX-internal).
The disk writer / manifest rewrite of that script is not part of this build.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _abi
from ._dev import ptr, stream_handle, to_device
from .mlx_weights import Q3_GROUP_SIZE, dequant_q3

FP4_EXPERT_BYTES = 18800640  # reference geometry: 3 x (2304 x 5120) FP4 + scales per expert


def parse_layers(arg: str) -> list[int]:
    """"20-23" -> [20..23]; "2,5,7" -> [2,5,7]; mixed lists allowed."""
    layers: list[int] = []
    for item in arg.split(","):
        lo, sep, hi = item.partition("-")
        if sep:
            layers.extend(range(int(lo), int(hi) + 1))
        else:
            layers.append(int(item))
    return layers


def parse_experts(arg: str | None, total: int = 384) -> list[int]:
    """None / "" -> every expert id; otherwise the same syntax as parse_layers."""
    return list(range(total)) if not arg else parse_layers(arg)


def quantize_q3(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Device f32 [rows, cols] -> (words int32-view [rows, cols*3/32], scales f16, biases f16)."""
    if w.dtype != torch.float32 or not w.is_cuda or w.dim() != 2:
        raise ValueError("quantize_q3 expects a 2-D float32 CUDA tensor")
    w = w.contiguous()
    rows, cols = w.shape
    if cols % Q3_GROUP_SIZE:
        raise ValueError(f"cols {cols} not a multiple of {Q3_GROUP_SIZE}")
    words = torch.empty((rows, cols * 3 // 32), dtype=torch.int32, device=w.device)
    scales = torch.empty((rows, cols // 64), dtype=torch.float16, device=w.device)
    biases = torch.empty_like(scales)
    _abi.call("ds_q3_quantize", ptr(w), rows, cols, ptr(words), ptr(scales), ptr(biases),
              stream_handle(w.device))
    return words, scales, biases


def convert_tensor(vals: np.ndarray, rows: int, cols: int, bits: int) -> tuple[bytes, bytes, bytes, float]:
    """f32 values -> (u32 word bytes, f16 scale bytes, f16 bias bytes, relative RMS error)."""
    if bits != 3:
        raise NotImplementedError("only 3-bit affine quantisation is implemented")
    w = to_device(np.asarray(vals, dtype=np.float32).reshape(rows, cols))
    words, scales, biases = quantize_q3(w)
    rt = dequant_q3(words, scales, biases)
    rt_scale = max(float(rt.abs().max()), 1e-9)
    err = w.double() - rt.double()
    rms = float(torch.sqrt(torch.mean(err * err))) / rt_scale
    return (words.cpu().numpy().view("<u4").tobytes(), scales.cpu().numpy().astype("<f2").tobytes(),
            biases.cpu().numpy().astype("<f2").tobytes(), rms)
