"""One weight sweep for up to two activation vectors at K=3840 (IronMule ironmule/qmv_shared.py:1-181).

`run_shared(w, scales, biases, vectors, out_features)` returns one [1, N] result per vector. On the B200 the
vectors are the rows of one qGEMM call (M = len(vectors)); the qGEMM is row-invariant, so each result is
bit-identical to the vector's own one-row call -- the property the reference's shared kernel keeps by
sharing the load and not the arithmetic.
"""
from __future__ import annotations

import torch

from . import kernel_registry

SIMD_SIZE = 32
NUM_SIMDGROUPS = 2
TARGET_K = 3840


def _kernel(width: int) -> kernel_registry.DeviceKernel:
    inputs = ["w", "scales", "biases"] + [f"x{v}" for v in range(width)] + ["shape"]
    return kernel_registry.build(f"qmv_k3840_shared_x{width}", source="qgemm_w4g64", input_names=inputs,
                                 output_names=[f"out{v}" for v in range(width)], ensure_row_contiguous=True,
                                 template={"width": width, "k": TARGET_K, "variant": "mma"})


SHARED = {width: _kernel(width) for width in (1, 2)}
_SHAPES: dict[tuple[int, int], torch.Tensor] = {}


def shape_array(in_features: int, out_features: int) -> torch.Tensor:
    key = (in_features, out_features)
    if key not in _SHAPES:
        _SHAPES[key] = torch.tensor([in_features, out_features], dtype=torch.int32)
    return _SHAPES[key]


def run_shared(w, scales, biases, vectors, out_features: int):
    """One weight sweep, `len(vectors)` independent results."""
    width = len(vectors)
    groups = (out_features + 7) // 8
    return SHARED[width](inputs=[w, scales, biases, *vectors, shape_array(TARGET_K, out_features)],
                         output_shapes=[(1, out_features)] * width, output_dtypes=[vectors[0].dtype] * width,
                         grid=(SIMD_SIZE, NUM_SIMDGROUPS * groups, 1), threadgroup=(SIMD_SIZE, NUM_SIMDGROUPS, 1))
