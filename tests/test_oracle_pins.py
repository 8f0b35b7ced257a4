"""The oracle pinned to the reference: the C restatement of the qmv arithmetic against the outputs of the
reference's own Metal kernel source (compiled for the CPU; fixtures in tests/golden/qmv_*.npz, made by
tests/golden/make_golden.py), plus the quantiser and bf16 helpers it builds on."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import bf16, qmv, quant

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = sorted(GOLDEN.glob("qmv_*.npz"))


def test_fixtures_exist():
    assert len(CASES) == 9


@pytest.mark.parametrize("path", CASES, ids=lambda p: p.stem)
@pytest.mark.parametrize("bf16_partials", [False, True])
def test_restatement_equals_the_reference_kernel_bit_for_bit(path, bf16_partials):
    d = np.load(path)
    y = qmv.qmv(d["wq"], d["scales"], d["biases"], d["x"], int(d["vpt"]), bf16_partials)
    want = d["y_bf1"] if bf16_partials else d["y_bf0"]
    assert np.array_equal(y, want)


@pytest.mark.parametrize("path", CASES, ids=lambda p: p.stem)
def test_reference_kernel_is_within_bf16_tolerance_of_float64(path):
    """Float sums (bf0) stay within 1e-2 max / 3e-3 mean of float64 (the output's own bf16 rounding is
    ~1.5e-3 mean); rounding every 4-term partial to bf16 (bf1) costs about ten times that."""
    d = np.load(path)
    ref = qmv.qmm_f64(d["wq"], d["scales"], d["biases"], d["x"])
    for key, max_rel, mean_rel in (("y_bf0", 1e-2, 3e-3), ("y_bf1", 2e-2, 2e-2)):
        err = np.abs(bf16.to_f32(d[key]) - ref)
        assert err.max() / np.abs(ref).max() <= max_rel
        assert err.mean() / np.abs(ref).mean() <= mean_rel


def test_bf16_round_trip_and_rounding():
    x = np.array([1.0, 1.00390625, 1.005859375, -2.5, 3.0e38, np.inf, -np.inf], dtype=np.float32)
    bits = bf16.from_f32(x)
    back = bf16.to_f32(bits)
    assert back[0] == 1.0 and back[3] == -2.5 and np.isinf(back[5]) and np.isinf(back[6])
    assert back[1] == 1.0  # a tie rounds to even
    assert back[2] == np.float32(1.0078125)
    assert np.isnan(bf16.to_f32(bf16.from_f32(np.array([np.nan], dtype=np.float32))))[0]


def test_quantiser_layout_and_error():
    rng = np.random.default_rng(3)
    w = bf16.round_f32(rng.normal(0, 0.02, (8, 256)).astype(np.float32))
    wq, s, b = quant.quantize(w)
    assert wq.shape == (8, 32) and wq.dtype == np.uint32 and s.shape == (8, 4) and b.shape == (8, 4)
    codes = quant.unpack(wq)
    assert codes.max() <= 15
    # low nibble first
    assert (wq[0, 0] & 0xF) == codes[0, 0] and ((wq[0, 0] >> 28) & 0xF) == codes[0, 7]
    deq = quant.dequantize(wq, s, b)
    step = np.repeat(bf16.to_f32(s), 64, axis=1)
    assert np.all(np.abs(deq - w) <= 0.5 * step + 2e-3 * np.abs(w) + 1e-6)


def test_quantiser_constant_group():
    w = np.full((1, 64), 0.25, dtype=np.float32)
    wq, s, b = quant.quantize(w)
    assert bf16.to_f32(s)[0, 0] == 0 and np.all(quant.unpack(wq) == 0)
    assert np.all(quant.dequantize(wq, s, b) == 0.25)


def test_restatement_refuses_uncovered_shapes():
    wq = np.zeros((1, 8), np.uint32)
    s = np.zeros((1, 1), np.uint16)
    with pytest.raises(ValueError):
        qmv.qmv(wq, s, s, np.zeros((1, 64), np.uint16), vpt=16)  # the fast path needs K % 512 == 0
