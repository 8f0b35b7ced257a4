"""TEST INFRASTRUCTURE ONLY: Philox4x32-10 counter-based RNG (Salmon, Moraes, Dror, Shaw, "Parallel random
numbers: as easy as 1, 2, 3", SC'11), vectorised in numpy.

Round: (hi0, lo0) = mulhilo(0xD2511F53, c0); (hi1, lo1) = mulhilo(0xCD9E8D57, c2);
       c = (hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0); then the key is bumped by (0x9E3779B9, 0xBB67AE85).
Ten rounds. `uniform(x)` maps an output word to [0, 1) exactly as the kernels do: (x >> 8) * 2^-24.

Stream layout used by the acceptance and sampling kernels: key = (seed low, seed high); counter =
(offset low, offset high, stream, draw) -- stream is the sequence (or sampled row), draw the use within it
(2i: accept test of draft i, 2i+1: resample after rejecting draft i, 2k: the bonus token after k accepts).
"""
from __future__ import annotations

import numpy as np

M0, M1 = np.uint64(0xD2511F53), np.uint64(0xCD9E8D57)
W0, W1 = np.uint32(0x9E3779B9), np.uint32(0xBB67AE85)
MASK = np.uint64(0xFFFFFFFF)


def philox4x32(counter, key, rounds: int = 10) -> np.ndarray:
    """counter uint32 [..., 4], key uint32 [..., 2] -> uint32 [..., 4]."""
    c = np.array(counter, dtype=np.uint32)
    k = np.array(key, dtype=np.uint32)
    c0, c1, c2, c3 = (c[..., i].astype(np.uint64) for i in range(4))
    k0, k1 = k[..., 0].astype(np.uint32), k[..., 1].astype(np.uint32)
    for r in range(rounds):
        if r:
            k0 = ((k0.astype(np.uint64) + np.uint64(W0)) & MASK).astype(np.uint32)
            k1 = ((k1.astype(np.uint64) + np.uint64(W1)) & MASK).astype(np.uint32)
        p0, p1 = M0 * c0, M1 * c2
        hi0, lo0 = p0 >> np.uint64(32), p0 & MASK
        hi1, lo1 = p1 >> np.uint64(32), p1 & MASK
        c0, c1, c2, c3 = (hi1 ^ c1 ^ k0.astype(np.uint64)), lo1, (hi0 ^ c3 ^ k1.astype(np.uint64)), lo0
    return np.stack([c0, c1, c2, c3], axis=-1).astype(np.uint32)


def uniform(word) -> np.ndarray:
    return (np.asarray(word, dtype=np.uint32) >> np.uint32(8)).astype(np.float64) * (1.0 / 16777216.0)


def stream_uniform(seed: int, offset: int, stream, draw) -> np.ndarray:
    """The uniform the kernels draw for (seed, offset, stream, draw); stream/draw broadcast."""
    stream, draw = np.broadcast_arrays(np.asarray(stream, dtype=np.uint64), np.asarray(draw, dtype=np.uint64))
    ctr = np.stack([np.full(stream.shape, offset & 0xFFFFFFFF), np.full(stream.shape, (offset >> 32) & 0xFFFFFFFF),
                    stream, draw], axis=-1).astype(np.uint32)
    key = np.broadcast_to(np.array([seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF], dtype=np.uint32),
                          stream.shape + (2,))
    return uniform(philox4x32(ctr, key)[..., 0])
