"""kernel_registry: the reference's naming contract (ironmule/kernel_registry.py:39-110), and the qmv
modules' kernels registered under it (tests/runtime/test_kernel_registry.py:89-142 restated)."""
from __future__ import annotations

import hashlib
import json

import pytest

from ironmule_b200 import kernel_registry as kr


def spec(**over):
    args = dict(source="qgemm_w4g64", input_names=["w", "x"], output_names=["out"])
    args.update(over)
    return kr.specification("t", **args)


def test_identifier_is_the_digest_of_the_canonical_specification():
    s = spec()
    canonical = json.dumps(s, sort_keys=True, separators=(",", ":"), ensure_ascii=True)
    assert kr.identifier(s) == "t_" + hashlib.sha256(canonical.encode()).hexdigest()[:16]
    assert len(kr.identifier(s).split("_")[-1]) == kr.IDENTIFIER_LENGTH == 16


def test_every_field_changes_the_name():
    base = kr.identifier(spec())
    for over in ({"source": "other"}, {"header": "h"}, {"input_names": ["w"]}, {"output_names": ["y"]},
                 {"ensure_row_contiguous": False}, {"atomic_outputs": True}, {"compile_options": {"a": 1}},
                 {"template": {"k": 1}}):
        assert kr.identifier(spec(**over)) != base


def test_same_spec_same_name_and_conflict_detection():
    a = kr.build("samebase", source="qgemm_w4g64", input_names=["w"], output_names=["o"])
    b = kr.build("samebase", source="qgemm_w4g64", input_names=["w"], output_names=["o"])
    assert a.name == b.name
    kr._REGISTRY[a.name] = dict(kr._REGISTRY[a.name], header="changed")
    with pytest.raises(kr.KernelSpecificationConflict):
        kr.build("samebase", source="qgemm_w4g64", input_names=["w"], output_names=["o"])
    del kr._REGISTRY[a.name]


def test_registered_is_a_copy():
    import ironmule_b200.qmv_k3840 as q  # noqa: F401

    got = kr.registered()
    assert any(name.startswith("qmv_k3840_") for name in got)
    got.clear()
    assert kr.registered()


def test_qmv_modules_register_distinct_kernels():
    import ironmule_b200.qmv_fast_shared as f
    import ironmule_b200.qmv_k3840 as q
    import ironmule_b200.qmv_shared as s
    import ironmule_b200.qmv_variant as v

    names = {q.PORT.name, q.K3840.name, s.SHARED[1].name, s.SHARED[2].name, v.kernel_for((4, 8)).name,
             v.kernel_for((2, 4)).name, *(k.name for k in f.KERNELS.values())}
    assert len(names) == 2 + 2 + 2 + 4


def test_kernel_call_validates_arity():
    k = kr.build("arity", source="qgemm_w4g64", input_names=["w", "scales", "biases", "x", "shape"],
                 output_names=["out"])
    with pytest.raises(ValueError):
        k(inputs=[1, 2], output_shapes=[(1, 8)], output_dtypes=[None])


def test_variant_gate():
    from ironmule_b200.qmv_variant import VariantGate

    gate = VariantGate()
    assert not gate.active and not gate.killed
    gate.open("eligible")
    assert gate.active and gate.reason == "eligible"
    gate.close("not eligible")
    assert not gate.active
    gate.open("again")
    gate.kill("fallback recorded")
    gate.open("anything")
    assert not gate.active and gate.killed
