"""3-bit affine (group 64) CPU oracle -- TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Reference semantics: ``w = scale * q + bias`` with q in 0..7 per 64-wide K
group, scale/bias stored as fp16 (src/deepseeker/mlx_forward.py:93-101;
scripts/requant_experts_3bit.py:69-83), payload shapes
``words [N, K*3/32] u32``, ``scales/biases [N, K/64] f16``
(src/deepseeker/mlx_weights.py:119-145).

The reference's bit packing is MLX-internal and MLX is not available, so the
bit layout below is BUILDER-DEFINED (parity unpinned at the bit level; the
shapes and the ValueError contract of ``unpack_int3_affine`` are pinned).

Bit layout of one 64-element group = 24 bytes = six little-endian u32 words:
  * words 0..3 ("low words"): word w holds the low two bits of elements
    16w..16w+15: bits [2j, 2j+2) <- element 16w+j and bits [16+2j, 18+2j) <-
    element 16w+8+j, for j = 0..7;
  * words 4..5 ("high words"): word 4+h holds bit 2 of elements 32h..32h+31:
    with w = 2h + v (v in {0,1}), bit 8v+j <- element 16w+j and bit 16+8v+j
    <- element 16w+8+j.
A shift and a mask of one low word and one high word give two 3-bit codes in
the two 16-bit halves of a register, which is what the CUDA decoders use.

Quantiser (builder-defined): per 64-group min/max in f32,
``scale16 = f16((max - min) / 7)``, ``bias16 = f16(min)``, and
``q = clamp(rint((w - f32(bias16)) / f32(scale16)), 0, 7)`` (q = 0 when
scale16 == 0), all f32 arithmetic round-to-nearest-even.
Dequant: ``f32(scale16) * q`` then ``+ f32(bias16)``: two roundings, no FMA.
"""
from __future__ import annotations

import numpy as np

GROUP = 64
BITS = 3
GROUP_BYTES = 24


def pack_codes(q: np.ndarray) -> np.ndarray:
    """codes [N, K] (0..7) -> words [N, K*3/32] u32 in the layout above."""
    q = np.asarray(q, dtype=np.uint32)
    n, k = q.shape
    assert k % GROUP == 0
    g = q.reshape(n, k // GROUP, 4, 16)           # [n, groups, w, 16]
    lo = g & 3
    hib = (g >> 2) & 1
    low_words = np.zeros((n, k // GROUP, 4), dtype=np.uint32)
    for j in range(8):
        low_words |= lo[..., j] << np.uint32(2 * j)
        low_words |= lo[..., 8 + j] << np.uint32(16 + 2 * j)
    high_words = np.zeros((n, k // GROUP, 2), dtype=np.uint32)
    for w in range(4):
        h, v = divmod(w, 2)
        for j in range(8):
            high_words[..., h] |= hib[..., w, j] << np.uint32(8 * v + j)
            high_words[..., h] |= hib[..., w, 8 + j] << np.uint32(16 + 8 * v + j)
    words = np.concatenate([low_words, high_words], axis=2)   # [n, groups, 6]
    return words.reshape(n, k // GROUP * 6)


def unpack_codes(words: np.ndarray, k: int) -> np.ndarray:
    """words [N, K*3/32] u32 -> codes [N, K] u8 (inverse of ``pack_codes``)."""
    words = np.asarray(words, dtype=np.uint32)
    n = words.shape[0]
    w6 = words.reshape(n, k // GROUP, 6)
    out = np.zeros((n, k // GROUP, 4, 16), dtype=np.uint32)
    for w in range(4):
        h, v = divmod(w, 2)
        lw = w6[..., w]
        hw = w6[..., 4 + h]
        for j in range(8):
            out[..., w, j] = ((lw >> np.uint32(2 * j)) & 3) | (((hw >> np.uint32(8 * v + j)) & 1) << 2)
            out[..., w, 8 + j] = ((lw >> np.uint32(16 + 2 * j)) & 3) | (((hw >> np.uint32(16 + 8 * v + j)) & 1) << 2)
    return out.reshape(n, k).astype(np.uint8)


def quantize(w: np.ndarray) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """[N, K] f32 -> (words u32 [N, K*3/32], scales f16 [N, K/64], biases f16 [N, K/64])."""
    w = np.asarray(w, dtype=np.float32)
    n, k = w.shape
    assert k % GROUP == 0
    g = w.reshape(n, k // GROUP, GROUP)
    mn = g.min(axis=2)
    mx = g.max(axis=2)
    scale16 = ((mx - mn) / np.float32(7.0)).astype(np.float32).astype(np.float16)
    bias16 = mn.astype(np.float16)
    s = scale16.astype(np.float32)[..., None]
    b = bias16.astype(np.float32)[..., None]
    with np.errstate(divide="ignore", invalid="ignore"):
        t = ((g - b).astype(np.float32) / s).astype(np.float32)
    q = np.where(s > 0, np.clip(np.rint(t), 0, 7), 0).astype(np.uint8)
    return pack_codes(q.reshape(n, k)), scale16, bias16


def dequant(words: np.ndarray, scales: np.ndarray, biases: np.ndarray) -> np.ndarray:
    """-> [N, K] f32: f32(scale) * q, then + f32(bias) (two roundings)."""
    scales = np.asarray(scales, dtype=np.float16)
    biases = np.asarray(biases, dtype=np.float16)
    n, groups = scales.shape
    k = groups * GROUP
    q = unpack_codes(words, k).astype(np.float32).reshape(n, groups, GROUP)
    s = scales.astype(np.float32)[..., None]
    b = biases.astype(np.float32)[..., None]
    prod = (s * q).astype(np.float32)
    return (prod + b).astype(np.float32).reshape(n, k)


def rel_rms(vals: np.ndarray, roundtrip: np.ndarray) -> float:
    """Quality metric of ``convert_tensor`` (requant_experts_3bit.py:74-78)."""
    rt_scale = max(float(np.abs(roundtrip).max()), 1e-9)
    err = np.asarray(vals, np.float64) - np.asarray(roundtrip, np.float64)
    return float(np.sqrt(np.mean(np.square(err))) / rt_scale)
