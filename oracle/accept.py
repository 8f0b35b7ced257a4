"""TEST INFRASTRUCTURE ONLY: acceptance rules on the CPU.

greedy_accept   the drafts equal to the target's argmax at their position, then the target's own token
                (IronMule ironmule/speculation.py:103-108).
row_stats       argmax (first index among equal maxima) and top-1 probability 1 / sum exp(l - l_max) per row
                (ironmule/ggml_engine.py:669-683).
"""
from __future__ import annotations

import numpy as np

from . import bf16


def greedy_accept(drafts, argmax) -> list[int]:
    n = 0
    while n < len(drafts) and drafts[n] == argmax[n]:
        n += 1
    return list(drafts[:n]) + [int(argmax[n])]


def row_stats(logits_bits: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    x = bf16.to_f32(logits_bits).astype(np.float64)
    idx = x.argmax(axis=-1)
    conf = 1.0 / np.exp(x - x.max(axis=-1, keepdims=True)).sum(axis=-1)
    return idx, conf
