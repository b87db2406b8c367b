"""FP4 (e2m1) / ue8m0 / e4m3 CPU oracle -- TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Restates:
  * ``FP4_TABLE`` / ``BLOCK``                      src/deepseeker/metal_fp4.py:21-26
  * ue8m0 decode (``_scale_lut_np``, ``decode_scales_u8m0``, ``decode_u8m0``)
                                                   metal_fp4.py:96-103, 134-136; mlx_weights.py:66-79
  * e2m1 dequant with f32 scales (``reference_dequant``)   metal_fp4.py:122-131
  * e2m1 dequant with raw u8 scales (``dequant_fp4_rowmajor``) mlx_weights.py:148-166
  * ``E4M3_TABLE`` and ``dequant_fp8_block``       mlx_weights.py:31-44, 82-89

plus the builder's FP4 quantiser for synthetic weights (the reference only
consumes pre-quantised checkpoints, so this rule is builder-defined):
per 32-element block ``e = ceil(log2(amax / 6))`` clamped to [-127, 127],
scale byte ``e + 127``, value ``w / 2^e`` rounded to the nearest e2m1 grid
point with ties going to the even code.
"""
from __future__ import annotations

import numpy as np

FP4_TABLE = np.array(
    [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
     0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0],
    dtype=np.float32,
)
BLOCK = 32


def u8m0_lut() -> np.ndarray:
    """256-entry ue8m0 table: byte b -> 2^(b-127) as f32, 0xFF -> NaN.

    b = 0 gives the f32 subnormal 2^-127 (metal_fp4.py:96-103).
    """
    bits = np.arange(256, dtype=np.int32)
    lut = np.exp2(bits - 127)
    lut[0xFF] = np.nan
    return lut.astype(np.float32)


_LUT = u8m0_lut()


def decode_u8m0(raw) -> np.ndarray:
    """ue8m0 bytes -> f32 powers of two (mlx_weights.py:66-79)."""
    raw = np.asarray(raw)
    if raw.dtype == np.uint8:
        return _LUT[raw]
    bits = raw.astype(np.int32)
    out = np.exp2(bits - 127).astype(np.float32)
    out[bits == 0xFF] = np.nan
    return out


def decode_scales_u8m0(raw: bytes) -> np.ndarray:
    """metal_fp4.py:134-136."""
    return _LUT[np.frombuffer(raw, dtype=np.uint8)]


def unpack_codes(packed: np.ndarray) -> np.ndarray:
    """Flat e2m1 codes, low nibble first (metal_fp4.py:124-129)."""
    raw = np.frombuffer(np.ascontiguousarray(packed).tobytes(), dtype=np.uint8)
    codes = np.empty(raw.size * 2, dtype=np.uint8)
    codes[0::2] = raw & 0x0F
    codes[1::2] = raw >> 4
    return codes


def dequant_f32_scales(packed: np.ndarray, scales_f32: np.ndarray) -> np.ndarray:
    """``reference_dequant`` (metal_fp4.py:122-131): LUT[nibble] * scale[e >> 5].

    Like the reference this requires ``scales_f32.size * 32 == n`` for the
    repeat to line up; the product is a single f32 multiply per element.
    """
    vals = FP4_TABLE[unpack_codes(packed)]
    rep = np.repeat(np.asarray(scales_f32, dtype=np.float32).reshape(-1), BLOCK)
    return vals * rep[: vals.size]


def dequant_u8_scales(packed: np.ndarray, raw_scales: np.ndarray) -> np.ndarray:
    """``dequant_fp4_rowmajor`` (mlx_weights.py:148-166): raw ue8m0 scale bytes,
    a tail block allowed (n need not be a multiple of 32)."""
    n = np.asarray(packed).size * 2
    n_scales = (n + 31) // 32
    raw_scales = np.asarray(raw_scales).reshape(-1)
    assert raw_scales.size == n_scales, (np.asarray(packed).size, raw_scales.size, n)
    vals = FP4_TABLE[unpack_codes(packed)]
    gain = decode_u8m0(raw_scales.astype(np.uint8))
    n_blocks = n // 32
    vals[: n_blocks * 32] *= np.repeat(gain[:n_blocks], 32)
    if n_blocks * 32 < n:
        vals[n_blocks * 32:] *= gain[n_blocks]
    return vals


# ---------------------------------------------------------------------------
# e4m3 (mlx_weights.py:31-44) and 32x32-block FP8 dequant (mlx_weights.py:82-89)

def _e4m3_table() -> np.ndarray:
    t = np.zeros(256, dtype=np.float32)
    for b in range(256):
        s = -1.0 if (b >> 7) & 1 else 1.0
        e = (b >> 3) & 0xF
        m = b & 0x7
        if e == 0xF and m == 0x7:
            t[b] = np.nan
        elif e == 0:
            t[b] = s * (m / 8.0) * 2.0 ** -6
        else:
            t[b] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return t


E4M3_TABLE = _e4m3_table()


def dequant_fp8_block(packed: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """[R, C] e4m3 bytes + [R/32, C/32] ue8m0 -> f32: value * scale[i//32, j//32]."""
    rows, cols = packed.shape
    assert rows % 32 == 0 and cols % 32 == 0
    assert scales.shape == (rows // 32, cols // 32)
    values = E4M3_TABLE[packed.astype(np.int64)]
    gain = np.repeat(np.repeat(decode_u8m0(scales.astype(np.uint8)), 32, axis=0), 32, axis=1)
    return values * gain


# ---------------------------------------------------------------------------
# builder's FP4 quantiser (synthetic weights only)



def quantize_fp4(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """[N, K] float -> (packed [N, K/2] u8, raw scales [N, K/32] u8).

    Block exponent e = ceil(log2(amax/6)) (0 for an all-zero block), clamped to
    [-127, 127]; codes = RNE of |w|/2^e onto the e2m1 magnitude grid, ties to
    the even code, saturating at 6; negative zero is stored as code 0.
    """
    w = np.asarray(w, dtype=np.float32)
    n, k = w.shape
    assert k % 32 == 0
    blocks = w.reshape(n, k // 32, 32).astype(np.float64)
    amax = np.abs(blocks).max(axis=2)
    with np.errstate(divide="ignore"):
        e = np.where(amax > 0, np.ceil(np.log2(amax / 6.0)), 0.0).astype(np.int64)
    # exact fix-up: smallest e with amax <= 6 * 2^e (guards log2 rounding)
    pos = amax > 0
    for _ in range(4):
        up = pos & (amax > np.ldexp(6.0, e))
        e = e + up
        down = pos & (amax <= np.ldexp(6.0, e - 1))
        e = e - down
    e = np.clip(e, -127, 127).astype(np.int32)
    scaled = blocks * np.ldexp(1.0, -e.astype(np.int64))[:, :, None]
    m = np.abs(scaled)
    # nearest e2m1 magnitude, ties to the even code: a tie at a midpoint goes
    # down when the lower code is even (strict >) and up when it is odd (>=)
    idx = ((m > 0.25).astype(np.int32) + (m >= 0.75) + (m > 1.25) + (m >= 1.75)
           + (m > 2.5) + (m >= 3.5) + (m > 5.0))
    sign = (scaled < 0) & (idx > 0)
    codes = (idx + 8 * sign).astype(np.uint8).reshape(n, k)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
    return packed, (e + 127).astype(np.uint8)


def dequant_matrix(packed: np.ndarray, raw_scales: np.ndarray) -> np.ndarray:
    """[N, K/2] u8 + [N, K/32] u8 -> [N, K] f32 (row-major, per row blocks)."""
    n = packed.shape[0]
    return dequant_u8_scales(packed.reshape(-1), raw_scales.reshape(-1)).reshape(n, -1)
