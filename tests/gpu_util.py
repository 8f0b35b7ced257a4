"""Helpers shared by the GPU tests: seeded MLX-affine cases built by the oracle, moved to the device."""
from __future__ import annotations

import numpy as np
import torch

from oracle import bf16, quant


def bf16_bits_to_torch(bits: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(device)


def torch_to_bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def u32_to_torch(a: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int32)).to(device)


def case(n: int, k: int, m: int, seed: int, sigma_w: float = 0.02):
    """Seeded W ~ N(0, sigma_w) rounded to bf16 and quantised; X ~ N(0, 1) in bf16 (host arrays)."""
    rng = np.random.default_rng(seed)
    w = bf16.round_f32(rng.normal(0.0, sigma_w, (n, k)).astype(np.float32))
    wq, s, b = quant.quantize(w)
    x = bf16.from_f32(rng.normal(0.0, 1.0, (m, k)).astype(np.float32))
    return wq, s, b, x


def to_device(wq, s, b, x, device):
    return (u32_to_torch(wq, device), bf16_bits_to_torch(s, device), bf16_bits_to_torch(b, device),
            bf16_bits_to_torch(x, device))


def rel_errors(got_bits: np.ndarray, want_bits: np.ndarray) -> tuple[float, float]:
    """(max |a-b| / max |b|, mean |a-b| / mean |b|) -- the reference's own probe metric
    (ironmule/cuda_native.py:253-268) and its mean."""
    a = bf16.to_f32(got_bits).astype(np.float64)
    b = bf16.to_f32(want_bits).astype(np.float64)
    err = np.abs(a - b)
    return float(err.max() / max(np.abs(b).max(), 1e-30)), float(err.mean() / max(np.abs(b).mean(), 1e-30))


MAX_REL, MEAN_REL = 1e-2, 1e-3  # bf16 tolerance of the qGEMM against the reference arithmetic
