"""Shared-weight matvec for the aligned projections K in (4096, 15360)
(IronMule ironmule/qmv_fast_shared.py:1-172): `run_fast(w, scales, biases, vectors, out_features, in_features)`.
On the B200 the same row-invariant qGEMM serves every K that is a multiple of 64; the supported set is kept
for call-site compatibility (a K outside it raises KeyError, as the reference's kernel table does).
"""
from __future__ import annotations

import torch

from . import kernel_registry

SIMD_SIZE = 32
NUM_SIMDGROUPS = 2
SUPPORTED_K = (4096, 15360)


def _kernel(k: int, width: int) -> kernel_registry.DeviceKernel:
    inputs = ["w", "scales", "biases"] + [f"x{v}" for v in range(width)] + ["shape"]
    return kernel_registry.build(f"qmv_fast_k{k}_x{width}", source="qgemm_w4g64", input_names=inputs,
                                 output_names=[f"out{v}" for v in range(width)], ensure_row_contiguous=True,
                                 template={"width": width, "k": k, "variant": "mma"})


KERNELS = {(k, width): _kernel(k, width) for k in SUPPORTED_K for width in (1, 2)}
_SHAPES: dict[tuple[int, int], torch.Tensor] = {}


def shape_array(in_features: int, out_features: int) -> torch.Tensor:
    key = (in_features, out_features)
    if key not in _SHAPES:
        _SHAPES[key] = torch.tensor([in_features, out_features], dtype=torch.int32)
    return _SHAPES[key]


def run_fast(w, scales, biases, vectors, out_features: int, in_features: int):
    """One weight sweep for `len(vectors)` requests on an aligned reduction length."""
    width = len(vectors)
    groups = (out_features + 7) // 8
    return KERNELS[(in_features, width)](
        inputs=[w, scales, biases, *vectors, shape_array(in_features, out_features)],
        output_shapes=[(1, out_features)] * width, output_dtypes=[vectors[0].dtype] * width,
        grid=(SIMD_SIZE, NUM_SIMDGROUPS * groups, 1), threadgroup=(SIMD_SIZE, NUM_SIMDGROUPS, 1))
