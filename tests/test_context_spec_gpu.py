"""Context speculation on the B200 (ironmule_b200.context_spec over engine.DeviceDraftEngine wrapping the target):
several requests verified together in one call per step, n-gram drafts from each request's own context; the
answers equal plain greedy decoding token for token (the reference's ggml step without a draft model,
ironmule/ggml_engine.py:1155-1343)."""
from __future__ import annotations

import pytest
import torch

from ironmule_b200 import context_spec, engine

pytestmark = pytest.mark.gpu


def tiny(seed, **kw):
    return engine.QuantModel(engine.PRESETS["tiny-target"], "cuda", seed=seed, sigma=0.08, max_ctx=256, **kw)


def test_context_speculation_equals_greedy(cuda):
    target = tiny(1, max_seqs=3)
    gen = torch.Generator().manual_seed(7)
    prompts = [[5, 9, 2, 7] * 6, torch.randint(0, 1000, (17,), generator=gen).tolist(), [42, 43]]
    limits = [40, 30, 25]
    tokens, stats = context_spec.context_generate(engine.DeviceDraftEngine(target), prompts, limits)
    solo = tiny(1)
    for p, n, got in zip(prompts, limits, tokens):
        assert got == engine.greedy_decode(solo, torch.tensor(p, device=cuda), n)
    assert stats["steps"] >= 1 and stats["rows"] >= stats["steps"]
