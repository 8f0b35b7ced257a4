"""GGUF files for the ggml path: a reader of the container format and device-resident Q4_K / Q6_K matrices served by
the k-quant matmul (`kernels.kq_gemv`, the B200 counterpart of the reference's generated kernels behind its llama.cpp
hook, ironmule/kernel_gen.py:58-862; the reference finds its Q4_K / Q6_K tensors in a GGUF file through llama.cpp's
own reader, kernel_gen.py:977-991).

Format (GGUF v2/v3, little-endian): magic "GGUF", version u32, tensor count u64, metadata count u64; metadata as
(string key, u32 value type, value); tensor infos as (string name, u32 dimension count, u64 dimensions innermost
first, u32 ggml type, u64 offset into the data section); the data section starts at the next multiple of
`general.alignment` (32 by default). A string is a u64 length and its bytes; an array a u32 element type, a u64 count
and the elements. A tensor of a ggml type this reader has no block size for (the IQ types, integer tensors, ...) stays
in the table with an unknown size: the file opens, and only asking for that tensor's bytes raises.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import numpy as np

MAGIC = b"GGUF"
# metadata value types
_SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}
_STRING, _ARRAY = 8, 9
# ggml tensor types: (elements per block, bytes per block)
TYPES = {0: (1, 4), 1: (1, 2), 2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 8: (32, 34), 9: (32, 36),
         10: (256, 84), 11: (256, 110), 12: (256, 144), 13: (256, 176), 14: (256, 210), 15: (256, 292),
         30: (1, 2)}
F32, F16, Q4_K, Q6_K, BF16 = 0, 1, 12, 14, 30


class GGUFError(ValueError):
    pass


@dataclass
class GGUFTensor:
    name: str
    type: int
    dims: tuple[int, ...]  # innermost first, as the file stores them
    offset: int            # absolute byte offset of the data in the file
    n_bytes: int | None    # None: a ggml type without a known block size

    @property
    def shape(self) -> tuple[int, ...]:
        """Row-major shape: outermost first (a [N rows, K] matrix for a weight)."""
        return tuple(reversed(self.dims))


class _Cursor:
    def __init__(self, buf: memoryview):
        self.buf, self.pos = buf, 0

    def take(self, n: int) -> memoryview:
        if self.pos + n > len(self.buf):
            raise GGUFError("truncated GGUF file")
        out = self.buf[self.pos:self.pos + n]
        self.pos += n
        return out

    def unpack(self, fmt: str):
        return struct.unpack(fmt, self.take(struct.calcsize(fmt)))[0]

    def string(self) -> str:
        n = self.unpack("<Q")
        return bytes(self.take(n)).decode("utf-8")

    def value(self, vtype: int) -> Any:
        if vtype in _SCALAR:
            return self.unpack(_SCALAR[vtype])
        if vtype == _STRING:
            return self.string()
        if vtype == _ARRAY:
            etype, count = self.unpack("<I"), self.unpack("<Q")
            if etype in _SCALAR and etype != 7:
                fmt = _SCALAR[etype]
                arr = np.frombuffer(self.take(count * struct.calcsize(fmt)), dtype=np.dtype(fmt))
                return arr.tolist()
            return [self.value(etype) for _ in range(count)]
        raise GGUFError(f"unknown metadata value type {vtype}")


class GGUFFile:
    """The metadata and tensor table of a GGUF file; tensor bytes are memory-mapped on demand."""

    def __init__(self, path: str | Path):
        self.path = Path(path)
        self._map = np.memmap(self.path, dtype=np.uint8, mode="r")
        cur = _Cursor(memoryview(self._map))
        if bytes(cur.take(4)) != MAGIC:
            raise GGUFError(f"{self.path}: not a GGUF file")
        self.version = cur.unpack("<I")
        if self.version not in (2, 3):
            raise GGUFError(f"{self.path}: GGUF version {self.version} (2 and 3 are read)")
        n_tensors, n_kv = cur.unpack("<Q"), cur.unpack("<Q")
        self.metadata: dict[str, Any] = {}
        for _ in range(n_kv):
            key = cur.string()
            self.metadata[key] = cur.value(cur.unpack("<I"))
        infos = []
        for _ in range(n_tensors):
            name = cur.string()
            nd = cur.unpack("<I")
            dims = tuple(cur.unpack("<Q") for _ in range(nd))
            ttype, offset = cur.unpack("<I"), cur.unpack("<Q")
            infos.append((name, ttype, dims, offset))
        self.alignment = int(self.metadata.get("general.alignment", 32))
        if self.alignment <= 0 or self.alignment & (self.alignment - 1):
            raise GGUFError(f"alignment {self.alignment} is not a power of two")
        data = -(-cur.pos // self.alignment) * self.alignment
        self.tensors: dict[str, GGUFTensor] = {}
        for name, ttype, dims, offset in infos:
            if ttype not in TYPES:
                self.tensors[name] = GGUFTensor(name, ttype, dims, data + offset, None)
                continue
            per, size = TYPES[ttype]
            count = int(np.prod(dims, dtype=np.int64)) if dims else 1
            if dims and dims[0] % per:
                raise GGUFError(f"{name}: {dims[0]} elements per row is not a whole number of blocks")
            n_bytes = count // per * size
            start = data + offset
            if start + n_bytes > len(self._map):
                raise GGUFError(f"{name}: data runs past the end of the file")
            self.tensors[name] = GGUFTensor(name, ttype, dims, start, n_bytes)

    def raw(self, name: str) -> np.ndarray:
        """The tensor's bytes (a read-only view of the file)."""
        t = self.tensors[name]
        if t.n_bytes is None:
            raise GGUFError(f"{name}: ggml type {t.type} is not read here")
        return self._map[t.offset:t.offset + t.n_bytes]

    def array(self, name: str) -> np.ndarray:
        """An F32 / F16 / BF16 tensor as float32 in its row-major shape."""
        t = self.tensors[name]
        raw = self.raw(name)
        if t.type == F32:
            out = raw.view(np.float32)
        elif t.type == F16:
            out = raw.view(np.float16).astype(np.float32)
        elif t.type == BF16:
            out = (raw.view(np.uint16).astype(np.uint32) << 16).view(np.float32)
        else:
            raise GGUFError(f"{name}: type {t.type} is quantized; use kquant_linear")
        return out.reshape(t.shape)


class KQuantLinear:
    """A Q4_K / Q6_K matrix resident on the device: y [B, N] = x [B, K] . W^T for 1-32 tokens (float32)."""

    def __init__(self, kind: int, weight: Any, n: int, k: int, device="cuda"):
        import torch

        if kind not in (Q4_K, Q6_K):
            raise GGUFError(f"type {kind}: only Q4_K (12) and Q6_K (14) run on the k-quant matmul")
        per, size = TYPES[kind]
        if k % per or len(weight) != n * (k // per) * size:
            raise GGUFError(f"{len(weight)} bytes are not {n} rows of {k // per} blocks")
        self.kind, self.n, self.k = kind, n, k
        self.w = torch.from_numpy(np.array(weight, dtype=np.uint8, copy=True)).to(device)

    def __call__(self, x, out=None):
        from . import kernels

        return kernels.kq_gemv(self.kind, self.w, x, self.n, out=out)


def kquant_linear(f: GGUFFile, name: str, device="cuda") -> KQuantLinear:
    """The Q4_K / Q6_K weight `name` of a GGUF file on the device ([N, K] with N = rows, K = the inner dimension)."""
    t = f.tensors[name]
    if len(t.dims) != 2:
        raise GGUFError(f"{name}: a matrix has two dimensions, not {len(t.dims)}")
    k, n = t.dims
    return KQuantLinear(t.type, f.raw(name), n, k, device)
