"""Per-head e4m3 quantiser oracle (test infrastructure only).

Restates ``quantize_fp8_e4m3_per_head``'s CPU path (F/inference/fused_kernels.py:823-834):

    scale[b, h] = max(amax_{s, d} |x[b, s, h, d]| / 448, 1e-12)        (fp32 division)
    q = e4m3fn(RTNE(clamp(x / scale, -448, 448)))                       (fp32 division)

in numpy, with the e4m3fn (1-4-3, bias 7, no infinities, max 448) round-to-nearest-even
encoding written out bit by bit, so the oracle does not depend on any library float8 cast.
"""

from __future__ import annotations

import numpy as np

FP8_MAX = np.float32(448.0)
SCALE_FLOOR = np.float32(1.0e-12)


def e4m3_encode(x: np.ndarray) -> np.ndarray:
    """RTNE fp32 -> e4m3fn bytes. Inputs must already lie in [-448, 448] (no NaN)."""

    x = np.asarray(x, dtype=np.float32)
    sign = (np.signbit(x)).astype(np.uint8) << 7
    a = np.abs(x).astype(np.float64)
    out = np.zeros(a.shape, dtype=np.uint8)
    sub = a < 2.0 ** -6
    # subnormals: value = m * 2^-9, m in [0, 8] (m == 8 is the smallest normal, code 0x08)
    m_sub = np.round(a[sub] / 2.0 ** -9).astype(np.int64)
    out[sub] = m_sub.astype(np.uint8)
    nrm = ~sub
    an = a[nrm]
    e = np.floor(np.log2(an)).astype(np.int64)
    # guard log2 rounding at exact powers of two
    e = np.where(an < 2.0 ** e, e - 1, e)
    e = np.where(an >= 2.0 ** (e + 1), e + 1, e)
    m = np.round((an / 2.0 ** e - 1.0) * 8.0).astype(np.int64)
    carry = m == 8
    e = np.where(carry, e + 1, e)
    m = np.where(carry, 0, m)
    out[nrm] = (((e + 7) << 3) | m).astype(np.uint8)
    return out | sign


def e4m3_decode(b: np.ndarray) -> np.ndarray:
    """e4m3fn bytes -> float32 (0x7F / 0xFF decode to NaN)."""

    b = np.asarray(b, dtype=np.uint8)
    sign = np.where(b & 0x80, -1.0, 1.0)
    e = (b >> 3) & 0xF
    m = (b & 0x7).astype(np.float64)
    val = np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * 2.0 ** (e.astype(np.int64) - 7))
    val = np.where((b & 0x7F) == 0x7F, np.nan, val)
    return (sign * val).astype(np.float32)


def quantize_fp8_e4m3_per_head(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """x [B, S, H, D] (bf16 values as float32) -> (e4m3 bytes [B, S, H, D], scale [B, H])."""

    x = np.asarray(x, dtype=np.float32)
    amax = np.abs(x).max(axis=(1, 3))
    scale = np.maximum(amax / FP8_MAX, SCALE_FLOOR).astype(np.float32)
    y = x / scale[:, None, :, None]
    y = np.clip(y, -FP8_MAX, FP8_MAX).astype(np.float32)
    return e4m3_encode(y), scale


def dequantize(q: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """e4m3 bytes [B, S, H, D] with scale [B, H] -> float32 values."""

    return e4m3_decode(q) * np.asarray(scale, dtype=np.float32)[:, None, :, None]


__all__ = ["e4m3_decode", "e4m3_encode", "dequantize", "quantize_fp8_e4m3_per_head"]
