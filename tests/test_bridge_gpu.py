"""The bridge (ironmule_b200.bridge) over the device decoders: more requests than slots, with different limits, an
end-of-generation token and a shared system prompt, served by continuous batching on a captured round. Slots start
and stop while other slots run, so a request's tokens depend only on its own prompt: every answer equals plain
greedy decoding cut at the first end token (the reference's `take`, ironmule/ggml_engine.py:1037-1056)."""
from __future__ import annotations

import pytest
import torch

from ironmule_b200 import bridge, engine

pytestmark = pytest.mark.gpu


def tiny(name, seed, b=1, rows=32):
    return engine.QuantModel(engine.PRESETS[name], "cuda", seed=seed, sigma=0.08, max_ctx=256, max_seqs=b,
                             max_rows=rows, max_logit_rows=rows)


def cut(tokens, eos):
    return tokens[:tokens.index(eos) + 1] if eos in tokens else tokens


@pytest.mark.parametrize("kind", ["linear", "linear-prefix", "tree-prefix"])
def test_bridge_answers_equal_greedy(cuda, kind):
    b = 2
    rows = 64 if kind.startswith("tree") else 32
    target, draft = tiny("tiny-target", 1, b, rows), tiny("tiny-draft", 2, b, rows)
    prefix = kind.endswith("prefix")
    if kind.startswith("tree"):
        dec = engine.TreeDecoder(target, draft, branch=(4, 2, 2), batch=b, prefix_cache=prefix)
    else:
        dec = engine.SpecDecoder(target, draft, k=4, batch=b, prefix_cache=prefix)
    gen = torch.Generator().manual_seed(17)
    system = torch.randint(0, 1000, (36,), generator=gen).tolist()
    ps = [system + torch.randint(0, 1000, (n,), generator=gen).tolist() for n in (5, 30, 2, 17, 9)]
    limits = [12, 20, 7, 15, 10]
    solo = tiny("tiny-target", 1)
    greedy = [engine.greedy_decode(solo, torch.tensor(p, device=cuda), lim) for p, lim in zip(ps, limits)]
    eos = greedy[1][6]
    br = bridge.DeviceBridge(dec, eos_ids=[eos])
    streamed = [[] for _ in ps]
    res = br.generate_many(ps, limits, on_tokens=[streamed[i].append for i in range(len(ps))])
    for i, r in enumerate(res):
        want = cut(greedy[i], eos)
        assert r.tokens == want and streamed[i] == want, i
        assert r.finish_reason == ("stop" if want[-1] == eos else "length"), i
    assert br.free_slots() == b
    again = br.generate_many(ps[:2], limits[:2])
    assert [r.tokens for r in again] == [cut(g, eos) for g in greedy[:2]]
    if prefix:
        # the system prompt's two full pages, and more of a prompt served before
        assert all(r.metrics["reused_prompt_tokens"] >= 32 for r in again)
        assert br.counters()["prefix"]["shared_tokens"] > 0
    br.close()
