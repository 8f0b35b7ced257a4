"""TEST INFRASTRUCTURE ONLY: ctypes wrapper of oracle/kquant_oracle.c, the CPU checker of the GGUF k-quant matmul.

`dequant` is ggml's float32 decoding of Q4_K / Q6_K blocks (the formats of ironmule/kernel_gen.py:68-97, :429-460);
`quantize_x` the activation rounding to 8 bits per 32 values (kernel_gen.py:86-97); `gemv` the device kernel's
arithmetic in its exact operation order (bit-exact target); `ref64` the float64 product used for error bounds.
`random_blocks` makes valid blocks from a seed (every bit pattern is a block; d and dmin are kept finite and small).
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
Q4_K, Q6_K = 12, 14
BLOCK_BYTES = {Q4_K: 144, Q6_K: 210}
_LIB = None
_P, _I = ctypes.c_void_p, ctypes.c_int64


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        path = HERE / "libkquant_oracle.so"
        if not path.exists():
            subprocess.run(["make", "-C", str(HERE), "libkquant_oracle.so"], check=True, capture_output=True)
        _LIB = ctypes.CDLL(str(path))
        _LIB.kq_dequant.argtypes = [ctypes.c_int, _P, _I, _P]
        _LIB.kq_quantize_x.argtypes = [_P, _I, _P, _P, _P]
        _LIB.kq_gemv.argtypes = [ctypes.c_int, _P, _I, _I, _P, _P, _P, _I, _P]
        _LIB.kq_ref64.argtypes = [ctypes.c_int, _P, _I, _I, _P, _I, _P]
    return _LIB


def _c(a: np.ndarray, dtype) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=dtype)


def random_blocks(kind: int, n_blocks: int, seed: int, scale: float = 2e-3) -> np.ndarray:
    """n_blocks valid blocks as uint8 [n_blocks, block bytes]: random quants and scales, f16 d (and dmin) near
    `scale`."""
    rng = np.random.default_rng(seed)
    size = BLOCK_BYTES[kind]
    blocks = rng.integers(0, 256, (n_blocks, size), dtype=np.uint8)
    d = (rng.uniform(0.5, 1.5, n_blocks) * scale).astype(np.float16).view(np.uint8).reshape(n_blocks, 2)
    if kind == Q4_K:
        dmin = (rng.uniform(0.5, 1.5, n_blocks) * scale).astype(np.float16).view(np.uint8).reshape(n_blocks, 2)
        blocks[:, 0:2], blocks[:, 2:4] = d, dmin
    else:
        blocks[:, 208:210] = d
    return blocks


def dequant(kind: int, blocks: np.ndarray) -> np.ndarray:
    b = _c(blocks, np.uint8).reshape(-1, BLOCK_BYTES[kind])
    out = np.empty(b.shape[0] * 256, dtype=np.float32)
    lib().kq_dequant(kind, b.ctypes.data, b.shape[0], out.ctypes.data)
    return out


def quantize_x(x: np.ndarray) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    x = _c(x, np.float32)
    n = x.size
    xq = np.empty(n, dtype=np.int8)
    dx = np.empty(n // 32, dtype=np.float32)
    xs = np.empty(n // 32, dtype=np.int32)
    lib().kq_quantize_x(x.ctypes.data, n, xq.ctypes.data, dx.ctypes.data, xs.ctypes.data)
    return xq.reshape(x.shape), dx, xs


def gemv(kind: int, w: np.ndarray, n: int, x: np.ndarray) -> np.ndarray:
    """The device kernel's y [B, N] (float32, bit-exact target) for x [B, K] float32."""
    x = _c(x, np.float32)
    b, k = x.shape
    w = _c(w, np.uint8)
    if w.size != n * (k // 256) * BLOCK_BYTES[kind]:
        raise ValueError("weights do not match N x K")
    xq, dx, xs = quantize_x(x)
    y = np.empty((b, n), dtype=np.float32)
    lib().kq_gemv(kind, w.ctypes.data, n, k, xq.ctypes.data, dx.ctypes.data, xs.ctypes.data, b, y.ctypes.data)
    return y


def ref64(kind: int, w: np.ndarray, n: int, x: np.ndarray) -> np.ndarray:
    x = _c(x, np.float64)
    b, k = x.shape
    w = _c(w, np.uint8)
    y = np.empty((b, n), dtype=np.float64)
    lib().kq_ref64(kind, w.ctypes.data, n, k, x.ctypes.data, b, y.ctypes.data)
    return y
