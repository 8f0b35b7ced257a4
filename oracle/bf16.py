"""TEST INFRASTRUCTURE ONLY: bfloat16 bit helpers for the oracle (numpy).

bf16 values travel as uint16 bit patterns. Conversion to bf16 rounds to nearest even; NaN stays NaN.
"""
from __future__ import annotations

import numpy as np


def to_f32(bits: np.ndarray) -> np.ndarray:
    """uint16 bf16 bit patterns -> float32."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def from_f32(x: np.ndarray) -> np.ndarray:
    """float32 -> uint16 bf16 bit patterns, round to nearest even."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    r = np.where(nan, (u >> 16) | 0x40, r)
    return r.astype(np.uint16)


def round_f32(x: np.ndarray) -> np.ndarray:
    """float32 rounded to the nearest bf16 value, returned as float32."""
    return to_f32(from_f32(x))
