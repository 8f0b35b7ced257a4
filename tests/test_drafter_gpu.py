"""The host Drafter (ironmule_b200.draft_model, the drop-in for ironmule/draft_model.py) driving a
draft model on the B200 through DeviceDraftEngine: the top token and its probability per logits row against the
host's scan of the same logits (ironmule/ggml_engine.py:669-683), drafts equal to the draft model's own greedy
continuation (also after a rejection trims its cache), and the host speculative loop with the confidence-stopped
draft lengths returning exactly plain greedy decoding's tokens."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from ironmule_b200 import draft_model as dm
from ironmule_b200 import engine

pytestmark = pytest.mark.gpu


def tiny(name, seed, **kw):
    return engine.QuantModel(engine.PRESETS[name], "cuda", seed=seed, sigma=0.08, max_ctx=256, **kw)


def host_pick(logits_row: torch.Tensor) -> tuple[int, float]:
    row = logits_row.float().cpu().numpy().astype(np.float64)
    top = int(np.flatnonzero(row == row.max())[0])
    return top, float(1.0 / np.exp(row - row[top]).sum())


def test_decode_conf_matches_the_host_scan(cuda):
    eng = engine.DeviceDraftEngine(tiny("tiny-draft", 2, max_seqs=2, max_rows=64))
    gen = torch.Generator().manual_seed(3)
    a = torch.randint(0, 1000, (45,), generator=gen).tolist()
    b = torch.randint(0, 1000, (6,), generator=gen).tolist()
    rows = [(t, j, 0, j == len(a) - 1) for j, t in enumerate(a)] + [(t, j, 1, j in (2, 5)) for j, t in enumerate(b)]
    got = eng._decode_conf(rows)
    assert eng.filled == [45, 6] and eng.forwards == 2
    ref = tiny("tiny-draft", 2)
    ta = torch.tensor(a, dtype=torch.int32, device=cuda)
    ref.prefill(ta[:-1])
    want = [host_pick(ref.logits_for(ta[-1:], len(a) - 1)[0])]
    lb = ref.logits_for(torch.tensor(b, dtype=torch.int32, device=cuda), 0)
    want += [host_pick(lb[2]), host_pick(lb[5])]
    assert [t for t, _ in got] == [t for t, _ in want]
    for (_, c), (_, w) in zip(got, want):
        assert abs(c - w) <= 1e-5 * w


def forced(drafter):
    drafter.stop.start = lambda running, sharers=1: True
    drafter.stop.more = lambda q, expected, spent, running, sharers: True
    return drafter


def test_drafts_are_the_draft_models_greedy_continuation(cuda):
    drafter = forced(dm.Drafter(engine.DeviceDraftEngine(tiny("tiny-draft", 2, max_seqs=2))))
    solo = tiny("tiny-draft", 2)
    gen = torch.Generator().manual_seed(9)
    context = torch.randint(0, 1000, (30,), generator=gen).tolist()
    out = drafter.draft({7: (context, 5)}, running=1)[7]
    assert out == engine.greedy_decode(solo, torch.tensor(context, device=cuda), 5)
    slot = drafter.slot_of[7]
    drafter.settle(7, used=5, accepted=1)  # the target kept one draft and put its own token after it
    assert drafter.held[slot] == context + out[:1]
    context = context + [out[0], (out[1] + 1) % 1000]
    out2 = drafter.draft({7: (context, 4)}, running=1)[7]
    assert out2 == engine.greedy_decode(solo, torch.tensor(context, device=cuda), 4)


@pytest.mark.parametrize("force", [False, True])
def test_drafter_generate_equals_greedy(cuda, force):
    target, solo = tiny("tiny-target", 1), tiny("tiny-target", 1)
    drafter = dm.Drafter(engine.DeviceDraftEngine(tiny("tiny-draft", 2)))
    if force:
        forced(drafter)
    prompt = torch.randint(0, 1000, (20,), generator=torch.Generator().manual_seed(5)).tolist()
    out, stats = engine.drafter_generate(target, drafter, prompt, 40, max_drafts=4)
    assert out == engine.greedy_decode(solo, torch.tensor(prompt, device=cuda), 40)
    if force:
        assert stats["drafted"] > 0
    assert stats["steps"] + stats["accepted"] == 40


def test_identical_draft_has_its_drafts_accepted(cuda):
    target, solo = tiny("tiny-target", 1), tiny("tiny-target", 1)
    drafter = forced(dm.Drafter(engine.DeviceDraftEngine(tiny("tiny-target", 1))))
    prompt = list(range(2, 30))
    out, stats = engine.drafter_generate(target, drafter, prompt, 30, max_drafts=4)
    assert out == engine.greedy_decode(solo, torch.tensor(prompt, device=cuda), 30)
    assert stats["accepted"] == stats["drafted"] and stats["steps"] == 6  # 5 tokens per step
