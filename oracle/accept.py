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


# ---- stochastic acceptance (the published speculative-sampling rule; no reference code exists) ----------------
def filtered_probs(logits_bits: np.ndarray, temperature: float, top_p: float) -> np.ndarray:
    """softmax(logits / T) restricted to the top-p set {v : l_v >= l*}, l* the largest logit whose set holds at
    least top_p of the mass (all ties at l* kept), renormalised; float64. NaN logits get probability 0."""
    l = bf16.to_f32(logits_bits).astype(np.float64)
    ok = ~np.isnan(l)
    m = l[ok].max()
    w = np.where(ok, np.exp((np.where(ok, l, m) - m) * np.float64(np.float32(1.0) / np.float32(temperature))), 0.0)
    if top_p < 1.0:
        total = w.sum()
        vals = np.unique(l[ok])[::-1]                      # distinct logits, descending
        mass = np.array([w[l == v].sum() for v in vals]) if vals.size < 4096 else None
        if mass is None:
            order = np.argsort(-l[ok], kind="stable")
            ls, ws = l[ok][order], w[ok][order]
            cum = np.cumsum(ws)
            j = int(np.searchsorted(cum, top_p * total, side="left"))
            j = min(j, ls.size - 1)
            cut = ls[j]
        else:
            cum = np.cumsum(mass)
            j = int(np.searchsorted(cum, top_p * total, side="left"))
            cut = vals[min(j, vals.size - 1)]
        w = np.where(ok & (l >= cut), w, 0.0)
    return w / w.sum()


def inverse_cdf(w: np.ndarray, u: float) -> int:
    """The first index whose cumulative weight exceeds u * total (index order)."""
    c = np.cumsum(w)
    idx = int(np.searchsorted(c, u * c[-1], side="right"))
    if idx >= w.size or w[idx] <= 0:
        idx = int(np.nonzero(w > 0)[0][-1]) if idx >= w.size else idx
    return idx


def sample_row(logits_bits, temperature, top_p, seed, offset, stream, draw) -> int:
    from .philox import stream_uniform

    p = filtered_probs(logits_bits, temperature, top_p)
    return inverse_cdf(p, float(stream_uniform(seed, offset, stream, draw)))


def accept_stochastic(target_bits, draft_bits, drafts, temperature, top_p, seed, offset, stream):
    """target_bits [k+1, V], draft_bits [k, V] (row i: the distribution draft i was sampled from).
    Returns (tokens, accepted, tests) with tests = [(u, p, q)] per tested draft."""
    from .philox import stream_uniform

    k = len(drafts)
    tests = []
    for i in range(k):
        p = filtered_probs(target_bits[i], temperature, top_p)
        q = filtered_probs(draft_bits[i], temperature, top_p)
        d = int(drafts[i])
        u = float(stream_uniform(seed, offset, stream, 2 * i))
        tests.append((u, p[d], q[d]))
        if not (u * q[d] < p[d]):
            r = np.maximum(p - q, 0.0)
            if r.sum() <= 0:
                r = p
            x = inverse_cdf(r, float(stream_uniform(seed, offset, stream, 2 * i + 1)))
            return list(map(int, drafts[:i])) + [x], i, tests
    p = filtered_probs(target_bits[k], temperature, top_p)
    x = inverse_cdf(p, float(stream_uniform(seed, offset, stream, 2 * k)))
    return list(map(int, drafts)) + [x], k, tests
