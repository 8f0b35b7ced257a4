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


def _gguf_bytes(version, kvs, tensors, alignment=None):
    """A GGUF file from the format: kvs [(key, type, value)], tensors [(name, dims innermost first, type, bytes)]."""
    def s(text):
        b = text.encode()
        return struct.pack("<Q", len(b)) + b

    def value(t, v):
        scalar = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q",
                  12: "<d"}
        if t in scalar:
            return struct.pack(scalar[t], v)
        if t == 8:
            return s(v)
        et, items = v
        return struct.pack("<IQ", et, len(items)) + b"".join(value(et, i) for i in items)

    if alignment is not None:
        kvs = kvs + [("general.alignment", 4, alignment)]
    out = b"GGUF" + struct.pack("<IQQ", version, len(tensors), len(kvs))
    for key, t, v in kvs:
        out += s(key) + struct.pack("<I", t) + value(t, v)
    align = alignment or 32
    offsets, off = [], 0
    for _, _, _, data in tensors:
        offsets.append(off)
        off += -(-len(data) // align) * align
    for (name, dims, t, _), o in zip(tensors, offsets):
        out += s(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        out += struct.pack("<IQ", t, o)
    out += bytes(-len(out) % align)
    for (_, _, _, data), o in zip(tensors, offsets):
        out += data + bytes(-(len(data)) % align)
    return out


def test_a_tensor_of_an_unknown_type_does_not_refuse_the_file(tmp_path):
    """An IQ4_XS tensor (ggml type 23: 256-value blocks of 136 bytes, no block size here) beside a Q4_K matrix: the
    file opens with both in its table; the Q4_K bytes read, and only asking for the IQ4_XS tensor's bytes raises."""
    rng = np.random.default_rng(4)
    q4k = rng.integers(0, 256, 2 * 144, dtype=np.uint8).tobytes()
    iq4 = rng.integers(0, 256, 3 * 136, dtype=np.uint8).tobytes()
    path = tmp_path / "mixed.gguf"
    path.write_bytes(_gguf_bytes(3, [("general.architecture", 8, "qwen3")],
                                 [("blk.0.ffn_down.weight", (256, 3), 23, iq4), ("blk.0.attn_q.weight", (256, 2), 12, q4k)]))
    f = gguf.GGUFFile(path)
    assert set(f.tensors) == {"blk.0.ffn_down.weight", "blk.0.attn_q.weight"}
    assert f.tensors["blk.0.ffn_down.weight"].n_bytes is None
    assert bytes(f.raw("blk.0.attn_q.weight")) == q4k
    for read in (f.raw, f.array, lambda name: gguf.kquant_linear(f, name, device="cpu")):
        with pytest.raises(gguf.GGUFError, match="not read here"):
            read("blk.0.ffn_down.weight")


def test_reader_alignment_v2_arrays_and_bf16(tmp_path):
    bf = (np.array([1.5, -2.0, 0.25], dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16).tobytes()
    q4 = kq.random_blocks(kq.Q4_K, 2, seed=3).tobytes()
    path = tmp_path / "edge.gguf"
    path.write_bytes(_gguf_bytes(
        2, [("a.bools", 9, (7, [True, False, True])), ("a.nested", 9, (9, [(4, [1, 2]), (4, [3])])),
            ("a.f64", 12, 0.125), ("a.i8", 1, -5), ("a.strs", 9, (8, ["x", "yz"]))],
        [("w", (256, 2), gguf.Q4_K, q4), ("b", (3,), gguf.BF16, bf)], alignment=64))
    f = gguf.GGUFFile(path)
    assert f.version == 2 and f.alignment == 64
    assert f.metadata["a.bools"] == [True, False, True] and f.metadata["a.nested"] == [[1, 2], [3]]
    assert f.metadata["a.f64"] == 0.125 and f.metadata["a.i8"] == -5 and f.metadata["a.strs"] == ["x", "yz"]
    assert f.tensors["w"].offset % 64 == 0 and f.tensors["b"].offset % 64 == 0
    assert f.raw("w").tobytes() == q4
    assert f.array("b").tolist() == [1.5, -2.0, 0.25]


def test_reader_refuses_malformed_tables(tmp_path):
    bad_type = tmp_path / "t.gguf"
    bad_type.write_bytes(_gguf_bytes(3, [], [("w", (256,), 99, bytes(8))]))
    with pytest.raises(gguf.GGUFError, match="type 99"):
        gguf.GGUFFile(bad_type).raw("w")  # the file opens; the tensor's bytes are refused
    ragged = tmp_path / "r.gguf"
    ragged.write_bytes(_gguf_bytes(3, [], [("w", (100, 2), gguf.Q4_K, bytes(288))]))
    with pytest.raises(gguf.GGUFError, match="whole number of blocks"):
        gguf.GGUFFile(ragged)
    odd = tmp_path / "a.gguf"
    odd.write_bytes(_gguf_bytes(3, [("general.alignment", 4, 48)], []))
    with pytest.raises(gguf.GGUFError, match="power of two"):
        gguf.GGUFFile(odd)
    badv = tmp_path / "v.gguf"
    badv.write_bytes(b"GGUF" + struct.pack("<IQQ", 3, 0, 1) + struct.pack("<Q", 1) + b"k" + struct.pack("<I", 42))
    with pytest.raises(gguf.GGUFError, match="value type 42"):
        gguf.GGUFFile(badv)


def test_kquant_linear_refuses_bad_shapes():
    with pytest.raises(gguf.GGUFError):
        gguf.KQuantLinear(gguf.F32, b"", 1, 256, device="cpu")
    with pytest.raises(gguf.GGUFError):
        gguf.KQuantLinear(gguf.Q4_K, bytes(100), 1, 256, device="cpu")
