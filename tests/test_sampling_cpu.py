"""The stochastic-acceptance oracle on the CPU: Philox4x32-10 against the Random123 known-answer vectors
(Salmon et al., SC'11), the top-p set, and the defining property of speculative sampling -- the emitted token
is distributed as the target's p whatever the draft's q (chi-square)."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import accept, bf16, philox


@pytest.mark.parametrize("ctr,key,want", [
    ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    ((0xFFFFFFFF,) * 4, (0xFFFFFFFF,) * 2, (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
     (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
])
def test_philox_known_answers(ctr, key, want):
    assert [int(x) for x in philox.philox4x32(ctr, key)] == list(want)


def test_uniform_range_and_mean():
    u = philox.stream_uniform(7, 3, np.arange(20000), 0)
    assert u.min() >= 0 and u.max() < 1 and abs(u.mean() - 0.5) < 0.01


def test_top_p_keeps_ties_and_the_smallest_sufficient_set():
    logits = bf16.from_f32(np.array([2.0, 1.0, 1.0, 0.0, -1.0], dtype=np.float32))
    p_all = accept.filtered_probs(logits, 1.0, 1.0)
    top = accept.filtered_probs(logits, 1.0, 0.5)
    assert top[0] > 0 and np.all(top[1:] == 0)          # the top token alone holds > 50%
    mid = accept.filtered_probs(logits, 1.0, p_all[0] + 0.01)
    assert mid[1] > 0 and mid[2] > 0 and mid[3] == 0     # the tie at 1.0 is kept whole
    assert np.isclose(mid.sum(), 1.0)


def chi2_ok(counts, probs, alpha=1e-3):
    from scipy.stats import chisquare

    keep = probs * counts.sum() >= 5
    exp = probs[keep] * counts.sum()
    obs = np.append(counts[keep], counts[~keep].sum())
    exp = np.append(exp, probs[~keep].sum() * counts.sum())
    if exp[-1] == 0:
        obs, exp = obs[:-1], exp[:-1]
    exp *= obs.sum() / exp.sum()
    return chisquare(obs, exp).pvalue > alpha


def test_speculative_sampling_emits_the_target_distribution():
    rng = np.random.default_rng(0)
    v = 12
    t = bf16.from_f32(rng.normal(0, 1.5, (2, v)).astype(np.float32))
    d = bf16.from_f32((bf16.to_f32(t[:1]) + rng.normal(0, 1.0, (1, v))).astype(np.float32))
    p0 = accept.filtered_probs(t[0], 0.7, 0.95)
    q0 = accept.filtered_probs(d[0], 0.7, 0.95)
    counts = np.zeros(v)
    for trial in range(4000):
        draft = accept.inverse_cdf(q0, float(philox.stream_uniform(11, trial, 0, 1000)))
        toks, _, _ = accept.accept_stochastic(t, d, [draft], 0.7, 0.95, 5, trial, 0)
        counts[toks[0]] += 1
    assert chi2_ok(counts, p0)
