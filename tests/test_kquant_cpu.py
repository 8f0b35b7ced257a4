"""GGUF k-quants on the CPU: the oracle's Q4_K / Q6_K decoding pinned bit for bit to ggml's own Python decoder (the
fixtures of tests/golden/make_kquant_golden.py), the oracle's kernel-order product against float64 and within the
reference's error bound (relative L2 error at most 1.25 x 6e-3 against float64, ironmule/kernel_gen.py:615, 1001,
1023), and the GGUF reader against what ggml's reader reports for a fixture file."""
import hashlib
import json
import struct
from pathlib import Path

import numpy as np
import pytest

from ironmule_b200 import gguf
from oracle import kquant as kq

GOLDEN = Path(__file__).resolve().parent / "golden"
BOUND = 1.25 * 6e-3


def rel_l2(y, ref):
    return float(np.sqrt(np.sum((y - ref) ** 2) / np.sum(ref ** 2)))


@pytest.mark.parametrize("kind,key", [(kq.Q4_K, "q4k"), (kq.Q6_K, "q6k")])
def test_dequant_equals_ggml(kind, key):
    g = np.load(GOLDEN / "kquant_golden.npz")
    mine = kq.dequant(kind, g[f"{key}_blocks"])
    assert np.array_equal(mine.view(np.uint32), g[f"{key}_values"].view(np.uint32))


@pytest.mark.parametrize("kind", [kq.Q4_K, kq.Q6_K])
def test_kernel_order_product(kind):
    n, k, b = 48, 2048, 5
    w = kq.random_blocks(kind, n * k // 256, seed=kind)
    x = np.random.default_rng(kind + 1).normal(0, 1, (b, k)).astype(np.float32)
    y = kq.gemv(kind, w, n, x)
    # against float64 over the same 8-bit activations: only fp32 rounding apart
    xq, dx, _ = kq.quantize_x(x)
    xd = xq.astype(np.float64) * np.repeat(dx.astype(np.float64), 32).reshape(b, k)
    same = kq.ref64(kind, w, n, xd)
    assert np.max(np.abs(y - same)) <= 2e-5 * np.max(np.abs(same))
    # against float64 over the unrounded activations: the reference's bound
    assert rel_l2(y, kq.ref64(kind, w, n, x)) <= BOUND
    # a token's result does not depend on the other tokens
    assert np.array_equal(kq.gemv(kind, w, n, x[2:3]), y[2:3])


def test_quantize_x_rounds_half_to_even_per_32():
    x = np.zeros(64, dtype=np.float32)
    x[0], x[1], x[2] = 127.0, 0.5, 1.5  # d = 1: 0.5 -> 0, 1.5 -> 2
    x[32:] = -2.0
    xq, dx, xs = kq.quantize_x(x)
    assert dx[0] == np.float32(1.0) and xq[1] == 0 and xq[2] == 2 and xs[0] == 127 + 0 + 2
    assert (xq[32:] == -127).all() and xs[1] == -127 * 32


def test_reader_matches_ggml_reader():
    want = json.loads((GOLDEN / "tiny_gguf.json").read_text())
    f = gguf.GGUFFile(GOLDEN / "tiny.gguf")
    assert f.alignment == want["alignment"] and f.version == 3
    for key, value in want["metadata"].items():
        got = f.metadata[key]
        assert got == pytest.approx(value) if isinstance(value, float) else got == value, key
    assert set(f.tensors) == set(want["tensors"])
    for name, t in want["tensors"].items():
        mine = f.tensors[name]
        assert (mine.type, list(mine.dims), mine.offset, mine.n_bytes) == (t["type"], t["dims"], t["offset"],
                                                                            t["n_bytes"]), name
        assert hashlib.sha256(f.raw(name).tobytes()).hexdigest() == t["sha256"], name
    assert f.tensors["blk.0.ffn_down.weight"].shape == (4, 512)
    assert np.allclose(f.array("output_norm.weight"), np.linspace(-1, 1, 512))
    assert f.array("token_embd.weight").tolist() == [[0, 1, 2], [3, 4, 5]]
    with pytest.raises(gguf.GGUFError):
        f.array("output.weight")


def test_reader_refusals(tmp_path):
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGML" + bytes(60))
    with pytest.raises(gguf.GGUFError, match="not a GGUF"):
        gguf.GGUFFile(bad)
    data = (GOLDEN / "tiny.gguf").read_bytes()
    cut = tmp_path / "cut.gguf"
    cut.write_bytes(data[:200])
    with pytest.raises(gguf.GGUFError, match="truncated"):
        gguf.GGUFFile(cut)
    short = tmp_path / "short.gguf"
    short.write_bytes(data[:-100])
    with pytest.raises(gguf.GGUFError, match="past the end"):
        gguf.GGUFFile(short)
    v9 = tmp_path / "v9.gguf"
    v9.write_bytes(data[:4] + struct.pack("<I", 9) + data[8:])
    with pytest.raises(gguf.GGUFError, match="version"):
        gguf.GGUFFile(v9)
