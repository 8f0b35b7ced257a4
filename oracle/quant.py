"""TEST INFRASTRUCTURE ONLY: MLX-affine 4-bit, group-64 quantisation in numpy.

Format (IronMule ironmule/cuda_native.py:54-56, ironmule/qmv_k3840.py:379-408): w uint32 [N, K/8] with
eight 4-bit codes per word, low nibble first; scales and biases bf16 [N, K/64]; w ~= scale * q + bias.

The quantiser is the per-group min/max recipe the benchmark configs name: scale = (max - min) / 15 and
bias = min, both rounded to bf16, then q = round((w - bias) / scale) clamped to 0..15, computed in float32
with the rounded scale and bias. A group whose scale rounds to 0 stores q = 0.
"""
from __future__ import annotations

import numpy as np

from . import bf16

GROUP = 64
BITS = 4


def quantize(w: np.ndarray) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """w float32 [N, K] (K % 64 == 0) -> (wq uint32 [N, K/8], scales u16 [N, K/64], biases u16 [N, K/64])."""
    w = np.asarray(w, dtype=np.float32)
    n, k = w.shape
    if k % GROUP:
        raise ValueError("K must be a multiple of 64")
    g = w.reshape(n, k // GROUP, GROUP)
    lo, hi = g.min(axis=2), g.max(axis=2)
    s_bits = bf16.from_f32((hi - lo) / np.float32(15.0))
    b_bits = bf16.from_f32(lo)
    s, b = bf16.to_f32(s_bits), bf16.to_f32(b_bits)
    safe = np.where(s == 0, np.float32(1.0), s)
    q = np.rint((g - b[:, :, None]) / safe[:, :, None])
    q = np.where(s[:, :, None] == 0, 0, q)
    q = np.clip(q, 0, 15).astype(np.uint32).reshape(n, k // 8, 8)
    shifts = (np.arange(8, dtype=np.uint32) * 4)[None, None, :]
    wq = np.bitwise_or.reduce(q << shifts, axis=2).astype(np.uint32)
    return wq, s_bits, b_bits


def unpack(wq: np.ndarray) -> np.ndarray:
    """uint32 [N, K/8] -> uint8 codes [N, K]."""
    wq = np.asarray(wq, dtype=np.uint32)
    shifts = (np.arange(8, dtype=np.uint32) * 4)[None, None, :]
    return ((wq[:, :, None] >> shifts) & 0xF).astype(np.uint8).reshape(wq.shape[0], -1)


def dequantize(wq: np.ndarray, s_bits: np.ndarray, b_bits: np.ndarray) -> np.ndarray:
    """float32 [N, K] = scale * q + bias, in float32 (no rounding of the product)."""
    q = unpack(wq).astype(np.float32)
    n, k = q.shape
    s = np.repeat(bf16.to_f32(s_bits), GROUP, axis=1)
    b = np.repeat(bf16.to_f32(b_bits), GROUP, axis=1)
    return s * q + b


def dequantize_bf16(wq: np.ndarray, s_bits: np.ndarray, b_bits: np.ndarray) -> np.ndarray:
    """bf16 bits [N, K]: the dequantised weight rounded to bf16 (how a quantised embedding row is read)."""
    return bf16.from_f32(dequantize(wq, s_bits, b_bits))
