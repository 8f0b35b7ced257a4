"""An alternative qGEMM configuration, installable per projection and gated at run time.

The drop-in counterpart of IronMule's `ironmule/qmv_variant.py` (VariantGate :57-79, kernel_for :81-96,
GatedVariantLinear :99-129, the byte-identity contract :132-142, install/uninstall :145-226). Same contract:
every candidate projection is run against the module it would replace on its own weights and a probe, and
is installed only if the two outputs are byte-identical; a single mismatch undoes the whole installation
and raises VariantUnsupported; installation is done once and a shared gate decides per call; a killed gate
never reopens; a shut gate calls the original module.

Geometries name kernel configurations of this build: a geometry with one SIMD group selects the CUDA-core
FMA kernel (v1), any other the warp-MMA kernel (v2) that the general path also uses. The reference's
qualified geometry, (4, 8), therefore maps to the general path's kernel and installs; the FMA kernel sums in
another order and is refused wherever its bytes differ.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch

from . import kernel_registry, qmv_k3840 as qmv
from .layers import QuantizedLinear

QUALIFIED_GEOMETRY = (4, 8)
QUALIFIED_ACTION_ID = "k3840_geometry_sg4_r8"
CORRECTNESS_CONTRACT = (
    "every admitted projection is byte-identical to the module it replaces on its own buffers "
    "before it is installed, and a projection that differs is left on the general path")


class VariantUnsupported(RuntimeError):
    """The variant is not admitted here. The general path stays in charge."""


@dataclass
class VariantGate:
    """One mutable boolean the installed projections read, and the reason it is shut."""

    active: bool = False
    killed: bool = False
    reason: str = "not activated"

    def open(self, reason: str) -> None:
        if self.killed:
            return
        self.active, self.reason = True, reason

    def close(self, reason: str) -> None:
        self.active, self.reason = False, reason

    def kill(self, reason: str) -> None:
        """Permanent for the life of this process."""
        self.active, self.killed, self.reason = False, True, reason


def kernel_for(geometry: tuple[int, int], fixed_k: int = qmv.TARGET_K) -> kernel_registry.DeviceKernel:
    simdgroups, results = geometry
    variant = "fma" if simdgroups == 1 else "mma"
    return kernel_registry.build(
        f"qmv_k{fixed_k}_sg{simdgroups}_r{results}", source="qgemm_w4g64",
        input_names=["w", "scales", "biases", "x", "shape"], output_names=["out"], ensure_row_contiguous=True,
        template={"fixed_k": fixed_k, "num_simdgroups": simdgroups, "results_per_simdgroup": results,
                  "variant": variant})


class GatedVariantLinear(torch.nn.Module):
    """An admitted projection that uses the variant only while its gate is open."""

    def __init__(self, source: QuantizedLinear, kernel, geometry: tuple[int, int], gate: VariantGate) -> None:
        super().__init__()
        self._source = source
        self._kernel = kernel
        self._gate = gate
        self.weight, self.scales, self.biases = source.weight, source.scales, source.biases
        self.group_size, self.bits = source.group_size, source.bits
        self.out_features = int(source.weight.shape[0])
        self._simdgroups = geometry[0]
        self._groups = self.out_features // (geometry[0] * geometry[1])
        self._shape = qmv.shape_array(qmv.TARGET_K, self.out_features)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        if not self._gate.active or len(shape) != 3 or shape[0] != 1 or shape[1] != 1:
            return self._source(x)
        out = self._kernel(inputs=[self.weight, self.scales, self.biases, x[0], self._shape],
                           output_shapes=[(1, self.out_features)], output_dtypes=[x.dtype],
                           grid=(qmv.SIMD_SIZE, self._simdgroups * self._groups, 1),
                           threadgroup=(qmv.SIMD_SIZE, self._simdgroups, 1))[0]
        return out[None]


def _identical(module: QuantizedLinear, kernel, geometry: tuple[int, int]) -> bool:
    """The contract, on this projection's own weights, before it is installed."""
    gen = torch.Generator(device=module.weight.device).manual_seed(0)
    probe = torch.randn((1, 1, qmv.TARGET_K), generator=gen, device=module.weight.device).to(torch.bfloat16)
    want = module(probe)
    got = GatedVariantLinear(module, kernel, geometry, VariantGate(active=True))(probe)
    torch.cuda.synchronize(module.weight.device)
    return bool(torch.equal(want.view(torch.int16), got.view(torch.int16)))


def install(model: torch.nn.Module, identity: Any,
            geometry: tuple[int, int] = QUALIFIED_GEOMETRY) -> tuple[VariantGate, dict[str, Any]]:
    """Admit the variant on this model or raise and leave it untouched. The gate comes back shut."""
    qmv._admit_environment(identity)
    simdgroups, results = geometry
    rows_per_group = simdgroups * results
    kernel = kernel_for(geometry)
    gate = VariantGate()
    admitted: list[str] = []
    declined: list[str] = []
    mismatched: list[str] = []

    def walk(parent: torch.nn.Module, prefix: str = "") -> None:
        for name, child in list(parent.named_children()):
            path = f"{prefix}.{name}" if prefix else name
            if isinstance(child, QuantizedLinear):
                if int(child.weight.shape[1]) * 32 // int(child.bits) != qmv.TARGET_K:
                    continue
                if not qmv._admit_projection(child) or int(child.weight.shape[0]) % rows_per_group:
                    declined.append(path)
                    continue
                if not _identical(child, kernel, geometry):
                    mismatched.append(path)
                    continue
                setattr(parent, name, GatedVariantLinear(child, kernel, geometry, gate))
                admitted.append(path)
            elif not isinstance(child, GatedVariantLinear):
                walk(child, path)

    walk(model)
    if mismatched:
        uninstall(model)
        raise VariantUnsupported(f"{len(mismatched)} projections were not byte-identical to the general path; "
                                 f"nothing is installed")
    if not admitted:
        raise VariantUnsupported("no projection met the admission conditions")
    return gate, {"admitted": len(admitted), "declined": len(declined), "mismatched": len(mismatched),
                  "admitted_paths": admitted, "declined_paths": declined,
                  "geometry": {"num_simdgroups": simdgroups, "results_per_simdgroup": results},
                  "action_id": QUALIFIED_ACTION_ID, "correctness_contract": CORRECTNESS_CONTRACT}


def uninstall(model: torch.nn.Module) -> int:
    """Put every installed projection back. Returns how many were restored."""
    restored = 0

    def walk(parent: torch.nn.Module) -> None:
        nonlocal restored
        for name, child in list(parent.named_children()):
            if isinstance(child, GatedVariantLinear):
                setattr(parent, name, child._source)
                restored += 1
            else:
                walk(child)

    walk(model)
    return restored
