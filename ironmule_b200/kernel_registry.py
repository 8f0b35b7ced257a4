"""One kernel name per specification, and never two specifications per name.

The drop-in counterpart of IronMule's `ironmule/kernel_registry.py:1-110`. The reference derives each
kernel's name from a SHA-256 digest over its whole specification, because MLX caches compiled kernels by
name (a stale-cache bug otherwise runs the wrong source). Here the kernels are precompiled into
libimspec.so, so nothing is compiled per name; the registry keeps the same contract anyway -- the same
`specification` / `identifier` / `build` / `registered` functions, the same digest, the same conflict
error -- so callers and their tests do not change, and a kernel's identity still covers everything that
decides what runs.

A specification's `source` names a libimspec program ("qgemm_w4g64") and its `template` the fixed
configuration (variant, epilogue, width, fixed K). `build` returns a `DeviceKernel`, called the way MLX
custom kernels are: `kernel(inputs=[...], output_shapes=[...], output_dtypes=[...], grid=..., threadgroup=...)`.
`grid` and `threadgroup` are accepted for call-site compatibility and ignored: each libimspec kernel picks
its own launch geometry for the B200.
"""
from __future__ import annotations

import hashlib
import json
from typing import Any, Callable, Mapping, Sequence

import torch

IDENTIFIER_LENGTH = 16


class KernelSpecificationConflict(RuntimeError):
    """One identifier was asked to stand for two different specifications."""


_REGISTRY: dict[str, dict[str, Any]] = {}
_PROGRAMS: dict[str, Callable] = {}


def specification(base: str, *, source: str, header: str = "",
                  input_names: Sequence[str], output_names: Sequence[str],
                  ensure_row_contiguous: bool = True, atomic_outputs: bool = False,
                  compile_options: Mapping[str, Any] | None = None,
                  template: Mapping[str, Any] | None = None) -> dict[str, Any]:
    """Everything that decides what runs, as one canonical mapping."""
    return {
        "base": base,
        "source": source,
        "header": header,
        "input_names": list(input_names),
        "output_names": list(output_names),
        "ensure_row_contiguous": bool(ensure_row_contiguous),
        "atomic_outputs": bool(atomic_outputs),
        "compile_options": dict(compile_options) if compile_options else None,
        "template": dict(template) if template else None,
    }


def identifier(spec: Mapping[str, Any]) -> str:
    """`<base>_<16 hex digits of sha256(canonical JSON)>`; the same specification always gets the same name."""
    canonical = json.dumps(spec, sort_keys=True, separators=(",", ":"), ensure_ascii=True)
    return f"{spec['base']}_{hashlib.sha256(canonical.encode()).hexdigest()[:IDENTIFIER_LENGTH]}"


def program(name: str):
    """Register the adapter that runs a libimspec program for kernels whose `source` is `name`."""
    def wrap(fn: Callable) -> Callable:
        _PROGRAMS[name] = fn
        return fn
    return wrap


class DeviceKernel:
    """A registered kernel: a libimspec program bound to a fixed configuration."""

    def __init__(self, name: str, spec: Mapping[str, Any]):
        self.name = name
        self.spec = dict(spec)
        self.input_names = list(spec["input_names"])
        self.output_names = list(spec["output_names"])
        self.template = dict(spec["template"] or {})

    def __call__(self, inputs: Sequence[torch.Tensor], output_shapes: Sequence[Sequence[int]],
                 output_dtypes: Sequence[torch.dtype], grid: Any = None, threadgroup: Any = None,
                 template: Any = None, **_: Any) -> list[torch.Tensor]:
        if len(inputs) != len(self.input_names):
            raise ValueError(f"{self.name}: {len(self.input_names)} inputs expected, {len(inputs)} given")
        if len(output_shapes) != len(self.output_names) or len(output_dtypes) != len(self.output_names):
            raise ValueError(f"{self.name}: {len(self.output_names)} outputs expected")
        named = dict(zip(self.input_names, inputs))
        if self.spec["ensure_row_contiguous"]:
            named = {k: (v.contiguous() if isinstance(v, torch.Tensor) else v) for k, v in named.items()}
        run = _PROGRAMS.get(self.spec["source"])
        if run is None:
            raise KeyError(f"{self.name}: no libimspec program named {self.spec['source']!r}")
        return run(named, [tuple(s) for s in output_shapes], list(output_dtypes), self.template)


def build(base: str, *, source: str, header: str = "",
          input_names: Sequence[str], output_names: Sequence[str],
          ensure_row_contiguous: bool = True, atomic_outputs: bool = False,
          compile_options: Mapping[str, Any] | None = None,
          template: Mapping[str, Any] | None = None) -> DeviceKernel:
    """Register a kernel under a name derived from its whole specification. Building the same
    specification twice gives the same name; a different specification always gets a different name,
    and a name that would stand for two specifications raises KernelSpecificationConflict."""
    spec = specification(base, source=source, header=header, input_names=input_names,
                         output_names=output_names, ensure_row_contiguous=ensure_row_contiguous,
                         atomic_outputs=atomic_outputs, compile_options=compile_options, template=template)
    name = identifier(spec)
    seen = _REGISTRY.get(name)
    if seen is not None and seen != spec:
        raise KernelSpecificationConflict(f"{name} already stands for a different specification")
    _REGISTRY[name] = spec
    return DeviceKernel(name, spec)


def registered() -> dict[str, dict[str, Any]]:
    """What this process has registered so far (a copy)."""
    return {name: dict(spec) for name, spec in _REGISTRY.items()}


@program("qgemm_w4g64")
def _run_qgemm(named: dict, output_shapes: list, output_dtypes: list, template: dict) -> list[torch.Tensor]:
    """The qmv family: inputs w, scales, biases, x or x0..x{width-1}, shape; one output per vector."""
    from . import kernels  # noqa: PLC0415 - keeps import of the registry free of the kernel library

    vectors = [named["x"]] if "x" in named else [named[f"x{v}"] for v in range(len(output_shapes))]
    k = vectors[0].shape[-1]
    fixed = template.get("k") or template.get("fixed_k")
    if fixed is not None and k != fixed:
        raise ValueError(f"kernel built for K={fixed}, called with K={k}")
    x = vectors[0].reshape(-1, k) if len(vectors) == 1 else torch.stack([v.reshape(k) for v in vectors])
    out = kernels.qgemm(x, named["w"], named["scales"], named["biases"], variant=template.get("variant", "auto"))
    if len(vectors) == 1:
        return [out.view(output_shapes[0])]
    return [out[i].view(output_shapes[i]) for i in range(len(vectors))]
