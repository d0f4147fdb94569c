"""Exact scalar formats in numpy: bf16 and e4m3 rounding (test infrastructure).

numpy has neither bfloat16 nor float8, so the oracle carries them as bit
images (uint16 / uint8) and rounds explicitly. Both conversions are
round-to-nearest-even, as the GPU's cvt.rn instructions and the reference's
compiled Triton kernels are.
"""
from __future__ import annotations

import numpy as np

E4M3_MAX = 448.0
FLT_MIN = np.float32(np.finfo(np.float32).tiny)


def bf16_bits_from_f32(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit image, round-to-nearest-even (NaN stays NaN)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        rounded = rounded.copy()
        rounded[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return rounded


def f32_from_bf16_bits(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 values to the nearest bf16 value, returned as fp32."""
    return f32_from_bf16_bits(bf16_bits_from_f32(x))


def f16_round(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def _e4m3_table() -> np.ndarray:
    codes = np.arange(256, dtype=np.uint32)
    sign = np.where(codes & 0x80, -1.0, 1.0)
    exp = (codes >> 3) & 0xF
    man = codes & 0x7
    val = np.where(exp == 0, man * 2.0 ** -9, (1.0 + man / 8.0) * 2.0 ** (exp.astype(np.float64) - 7))
    val = sign * val
    val[(codes & 0x7F) == 0x7F] = np.nan
    return val.astype(np.float32)


E4M3_VALUES = _e4m3_table()


def e4m3_to_f32(codes: np.ndarray) -> np.ndarray:
    return E4M3_VALUES[np.asarray(codes, dtype=np.uint8)]


def e4m3_from_f32(x: np.ndarray) -> np.ndarray:
    """fp32 -> e4m3 (fn) code, round-to-nearest-even, saturating to +-448."""
    x = np.asarray(x, dtype=np.float32).astype(np.float64)
    sign = np.signbit(x)
    a = np.minimum(np.abs(x), E4M3_MAX)
    code = np.zeros(a.shape, dtype=np.int64)
    normal = a >= 2.0 ** -6
    # Normal range: exponent e = floor(log2 a); 3-bit mantissa, RNE via rint.
    _, e = np.frexp(np.where(normal, a, 1.0))
    e = e - 1
    q = np.rint(np.where(normal, a, 0.0) * np.exp2(3.0 - e)).astype(np.int64)  # in [8, 16]
    carry = q == 16
    e = np.where(carry, e + 1, e)
    q = np.where(carry, 8, q)
    code = np.where(normal, ((e + 7) << 3) | (q - 8), code)
    sub = ~normal
    qs = np.rint(np.where(sub, a, 0.0) * 2.0 ** 9).astype(np.int64)  # 0..8; 8 == min normal
    code = np.where(sub, qs, code)
    code = np.minimum(code, 0x7E)  # satfinite: never the NaN code
    code = np.where(np.isnan(x), 0x7F, code)
    return (code | np.where(sign, 0x80, 0)).astype(np.uint8)


def e4m3_round(x: np.ndarray) -> np.ndarray:
    return e4m3_to_f32(e4m3_from_f32(x))


def fdiv(a, b) -> np.ndarray:
    """IEEE fp32 division."""
    return (np.asarray(a, dtype=np.float32) / np.asarray(b, dtype=np.float32)).astype(np.float32)
