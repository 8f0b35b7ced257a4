"""TEST INFRASTRUCTURE ONLY: ctypes wrapper of oracle/qmv_oracle.c (the reference's qmv arithmetic in C).

`qmv(...)` follows IronMule's Metal qmv kernels lane by lane (ironmule/qmv_k3840.py:62-244 with vpt=8;
ironmule/qmv_fast_shared.py:30-131 with vpt=16); `qmm_f64(...)` is a float64-accumulated dequantised
product used as the tolerance reference. `emu(...)` calls the reference's own Metal source compiled for
the CPU (oracle/_ref, built by oracle/build_ref.py in the container that holds the reference tree).
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
_LIB = None
_EMU: dict[int, ctypes.CDLL] = {}
_P = ctypes.c_void_p
_I = ctypes.c_int64


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        path = HERE / "libqmv_oracle.so"
        if not path.exists():
            subprocess.run(["make", "-C", str(HERE), "libqmv_oracle.so"], check=True, capture_output=True)
        _LIB = ctypes.CDLL(str(path))
        _LIB.oracle_qmv_w4g64.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I, ctypes.c_int, ctypes.c_int]
        _LIB.oracle_qmm_f64.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I]
        _LIB.oracle_qmm_fast.argtypes = [_P, _P, _P, _P, _P, _I, _I, _I]
    return _LIB


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def qmv(wq, s, b, x, vpt: int = 8, bf16_partials: bool = False) -> np.ndarray:
    """bf16 bits y [M, N] for x bf16 bits [M, K]."""
    wq = np.ascontiguousarray(wq, dtype=np.uint32)
    s = np.ascontiguousarray(s, dtype=np.uint16)
    b = np.ascontiguousarray(b, dtype=np.uint16)
    x = np.ascontiguousarray(x, dtype=np.uint16)
    if x.ndim == 1:
        x = x[None]
    m, k = x.shape
    n = wq.shape[0]
    y = np.zeros((m, n), dtype=np.uint16)
    rc = lib().oracle_qmv_w4g64(_ptr(wq), _ptr(s), _ptr(b), _ptr(x), _ptr(y), m, n, k, vpt, int(bf16_partials))
    if rc:
        raise ValueError(f"shape not covered by the vpt={vpt} arithmetic: K={k}")
    return y


def qmm_f64(wq, s, b, x) -> np.ndarray:
    """float32 [M, N] = x . (scale*q + bias)^T accumulated in float64."""
    wq = np.ascontiguousarray(wq, dtype=np.uint32)
    s = np.ascontiguousarray(s, dtype=np.uint16)
    b = np.ascontiguousarray(b, dtype=np.uint16)
    x = np.ascontiguousarray(x, dtype=np.uint16)
    if x.ndim == 1:
        x = x[None]
    m, k = x.shape
    out = np.zeros((m, wq.shape[0]), dtype=np.float32)
    lib().oracle_qmm_f64(_ptr(wq), _ptr(s), _ptr(b), _ptr(x), _ptr(out), m, wq.shape[0], k)
    return out


def emu(name: str, wq, s, b, x, bf16_partials: bool = False) -> np.ndarray:
    """Run the reference's own Metal kernel `name` (compiled for the CPU) over the rows of x.
    Kernels of width 2 take two rows per call, as the reference's shared kernels do."""
    flag = int(bf16_partials)
    if flag not in _EMU:
        path = HERE / "_ref" / f"libmlx_qmv_emu_bf{flag}.so"
        if not path.exists():
            raise FileNotFoundError(f"{path} missing: run `python oracle/build_ref.py` where the reference is")
        _EMU[flag] = ctypes.CDLL(str(path))
    fn = getattr(_EMU[flag], f"emu_{name}")
    fn.argtypes = [_P, _P, _P, _P, _P, ctypes.c_int, ctypes.c_int]
    wq = np.ascontiguousarray(wq, dtype=np.uint32)
    s = np.ascontiguousarray(s, dtype=np.uint16)
    b = np.ascontiguousarray(b, dtype=np.uint16)
    x = np.ascontiguousarray(x, dtype=np.uint16)
    if x.ndim == 1:
        x = x[None]
    m, k = x.shape
    n = wq.shape[0]
    width = 2 if name.endswith("_x2") else 1
    if m % width:
        raise ValueError("a width-2 kernel takes rows in pairs")
    y = np.zeros((m, n), dtype=np.uint16)
    for r in range(0, m, width):
        xr = np.ascontiguousarray(x[r:r + width])
        yr = np.zeros((width, n), dtype=np.uint16)
        fn(_ptr(wq), _ptr(s), _ptr(b), _ptr(xr), _ptr(yr), k, n)
        y[r:r + width] = yr
    return y


def qmm_fast(wq, s, b, x) -> np.ndarray:
    """bf16 bits y [M, N]: dequantise-and-dot in float32 (the timed CPU baseline's projection)."""
    x = np.ascontiguousarray(x, dtype=np.uint16)
    if x.ndim == 1:
        x = x[None]
    m, k = x.shape
    y = np.zeros((m, wq.shape[0]), dtype=np.uint16)
    rc = lib().oracle_qmm_fast(_ptr(np.ascontiguousarray(wq)), _ptr(np.ascontiguousarray(s)),
                               _ptr(np.ascontiguousarray(b)), _ptr(x), _ptr(y), m, wq.shape[0], k)
    if rc:
        raise ValueError("qmm_fast: unsupported shape")
    return y
