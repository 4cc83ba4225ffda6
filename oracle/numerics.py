"""Rounding helpers for the CPU oracle (test infrastructure only).

numpy has IEEE binary16 (``np.float16``) but no bfloat16, so bf16 arrays are
carried as their uint16 bit patterns and converted here with an explicit
round-to-nearest-even, which is what ``torch`` does for ``float -> bfloat16``.
"""
from __future__ import annotations

import numpy as np

F16 = "f16"
BF16 = "bf16"
F32 = "f32"

DTYPES = (F16, BF16, F32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit pattern, round-to-nearest-even, NaN kept quiet."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    out = rounded.astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        out[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return out


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def to_f32(a: np.ndarray, dtype: str) -> np.ndarray:
    """Widen an oracle array of ``dtype`` to float32 (exact)."""
    if dtype == BF16:
        return bf16_bits_to_f32(a)
    return np.asarray(a).astype(np.float32)


def from_f32(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to ``dtype`` (RNE); bf16 comes back as uint16 bits."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == F16:
        with np.errstate(over="ignore"):
            return x.astype(np.float16)
    if dtype == BF16:
        return f32_to_bf16_bits(x)
    if dtype == F32:
        return x.copy()
    raise ValueError(f"unknown dtype {dtype!r}")


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to ``dtype`` and widen back to float32."""
    return to_f32(from_f32(x, dtype), dtype)


def raw_bytes(a: np.ndarray) -> bytes:
    return np.ascontiguousarray(a).tobytes()
