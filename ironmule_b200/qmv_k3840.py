"""The K=3840 quantised matrix-vector path, behind an admission gate.

The drop-in counterpart of IronMule's `ironmule/qmv_k3840.py`: the same names (`PORT`, `K3840`,
`shape_array`, `run`, `K3840QuantizedLinear`, `enable`, `disable`, `K3840Unsupported`) and the same
contract -- admission is checked once at load and either admits projections or raises and leaves the model
untouched; a projection that was not admitted, or an input that is not a single-token decode, keeps the
module's general path.

What differs is what runs: both paths are the B200 qGEMM (`kernels.qgemm`). The reference admits only the
exact machine its Metal kernel was qualified on (hardware fingerprint, MLX versions, model identity,
ironmule/qmv_k3840.py:345-376); here admission requires a CUDA device of compute capability 10.x (B200),
libimspec loaded, and a model identity. Projection admission is the reference's: 4 bits, group 64, K=3840,
bf16 scales and biases, uint32 codes, exact buffer sizes (ironmule/qmv_k3840.py:379-408).
"""
from __future__ import annotations

from typing import Any

import torch

from . import kernel_registry
from .layers import QuantizedLinear


class K3840Unsupported(RuntimeError):
    """The candidate is not admitted here. The general path stays in charge."""


TARGET_K = 3840
SIMD_SIZE = 32
NUM_SIMDGROUPS = 2
RESULTS_PER_SIMDGROUP = 4
GROUP_SIZE = 64
VERIFIED_BITS = 4
VERIFIED_GROUP_SIZE = 64
VERIFIED_DTYPE = "bfloat16"
REQUIRED_CAPABILITY_MAJOR = 10


def _kernel(name: str, fixed_k: int | None) -> kernel_registry.DeviceKernel:
    return kernel_registry.build(
        name, source="qgemm_w4g64", input_names=["w", "scales", "biases", "x", "shape"], output_names=["out"],
        ensure_row_contiguous=True, template={"fixed_k": fixed_k, "variant": "mma"})


PORT = _kernel("qmv_port", None)
K3840 = _kernel("qmv_k3840", TARGET_K)

_SHAPES: dict[tuple[int, int], torch.Tensor] = {}


def shape_array(in_features: int, out_features: int) -> torch.Tensor:
    """One shared (K, N) constant per geometry."""
    key = (in_features, out_features)
    cached = _SHAPES.get(key)
    if cached is None:
        cached = torch.tensor([in_features, out_features], dtype=torch.int32)
        _SHAPES[key] = cached
    return cached


def run(kernel, w, scales, biases, x, out_features: int, in_features: int):
    """One decode row: y [1, N] for x [1, K] (or [K])."""
    groups = (out_features + 7) // 8
    return kernel(inputs=[w, scales, biases, x, shape_array(in_features, out_features)],
                  output_shapes=[(1, out_features)], output_dtypes=[x.dtype],
                  grid=(SIMD_SIZE, NUM_SIMDGROUPS * groups, 1), threadgroup=(SIMD_SIZE, NUM_SIMDGROUPS, 1))[0]


class K3840QuantizedLinear(torch.nn.Module):
    """An admitted projection: single-token decode goes through K3840, anything else through the source
    module, on the very same buffers."""

    def __init__(self, source: QuantizedLinear) -> None:
        super().__init__()
        self._source = source
        self.weight, self.scales, self.biases = source.weight, source.scales, source.biases
        self.group_size, self.bits = source.group_size, source.bits
        self.out_features = int(source.weight.shape[0])

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        if len(shape) != 3 or shape[0] != 1 or shape[1] != 1:
            return self._source(x)
        return run(K3840, self.weight, self.scales, self.biases, x[0], self.out_features, TARGET_K)[None]


def _admit_environment(identity: Any) -> None:
    """Checked once, at load."""
    from . import _lib  # noqa: PLC0415

    if not torch.cuda.is_available():
        raise K3840Unsupported("no CUDA device")
    major, minor = torch.cuda.get_device_capability()
    if major != REQUIRED_CAPABILITY_MAJOR:
        raise K3840Unsupported(f"built for compute capability 10.x (B200), found {major}.{minor}")
    try:
        _lib.load()
    except _lib.KernelLibraryMissing as exc:
        raise K3840Unsupported(str(exc)) from exc
    if identity is None:
        raise K3840Unsupported("no model identity available; the candidate fails closed")


def _admit_projection(module: QuantizedLinear) -> bool:
    if int(module.bits) != VERIFIED_BITS or int(module.group_size) != VERIFIED_GROUP_SIZE:
        return False
    if int(module.weight.shape[1]) * 32 // int(module.bits) != TARGET_K:
        return False
    out_features = int(module.weight.shape[0])
    if out_features % (NUM_SIMDGROUPS * RESULTS_PER_SIMDGROUP):
        return False
    for array in (module.scales, module.biases):
        if str(array.dtype).rsplit(".", 1)[-1] != VERIFIED_DTYPE:
            return False
    if module.weight.dtype not in (torch.int32, torch.uint32):
        return False
    if int(module.scales.shape[1]) != TARGET_K // VERIFIED_GROUP_SIZE or module.scales.shape != module.biases.shape:
        return False
    expected = ((module.weight, out_features * (TARGET_K * VERIFIED_BITS // 32) * 4),
                (module.scales, out_features * (TARGET_K // VERIFIED_GROUP_SIZE) * 2),
                (module.biases, out_features * (TARGET_K // VERIFIED_GROUP_SIZE) * 2))
    return all(a.is_contiguous() and a.numel() * a.element_size() == size for a, size in expected)


def _replace(module: torch.nn.Module, admitted: list[str], skipped: list[str], prefix: str = "") -> None:
    for name, child in list(module.named_children()):
        path = f"{prefix}.{name}" if prefix else name
        if isinstance(child, QuantizedLinear):
            if int(child.weight.shape[1]) * 32 // int(child.bits) != TARGET_K:
                continue
            if _admit_projection(child):
                setattr(module, name, K3840QuantizedLinear(child))
                admitted.append(path)
            else:
                skipped.append(path)
        elif not isinstance(child, K3840QuantizedLinear):
            _replace(child, admitted, skipped, path)


def _restore(module: torch.nn.Module, restored: list[str], prefix: str = "") -> None:
    for name, child in list(module.named_children()):
        path = f"{prefix}.{name}" if prefix else name
        if isinstance(child, K3840QuantizedLinear):
            setattr(module, name, child._source)
            restored.append(path)
        else:
            _restore(child, restored, path)


def disable(model: torch.nn.Module) -> int:
    """Put every admitted projection back on its original module. Returns how many."""
    restored: list[str] = []
    _restore(model, restored)
    return len(restored)


def enable(model: torch.nn.Module, identity: Any) -> dict[str, Any]:
    """Admit the candidate on this model, or raise and leave it untouched."""
    _admit_environment(identity)
    admitted: list[str] = []
    skipped: list[str] = []
    _replace(model, admitted, skipped)
    if not admitted:
        raise K3840Unsupported("no projection met the admission conditions")
    return {"admitted": len(admitted), "declined": len(skipped), "admitted_paths": admitted,
            "declined_paths": skipped, "device": torch.cuda.get_device_name()}
