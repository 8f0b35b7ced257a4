"""Context speculation over the device engine: the reference's ggml step with no draft model
(ironmule/ggml_engine.py:1155-1343, the bridge's default "speculation": "context"). Each step, every running
request offers the tokens that followed the last repeat of its own context's suffix (`speculation.NgramIndex`, and
other requests' finished answers through `CollectiveIndex` when its own offer is short), the policy chooses how many
drafts each verifies (`StepPolicy` by default: one call priced by its rows), one call verifies every request's last
token and drafts, `accept` keeps the agreed prefix and the target's own token, the policy learns the step's price and
each bucket's acceptance, and the rejected positions are dropped from the request's cache.

`engine` is the reference engine protocol the draft model also uses (`_decode_conf`, `eog`,
`L.llama_memory_seq_rm`, `memory`, `seqs`, plus `seq_ctx` and `max_rows`): `engine.DeviceDraftEngine` over the
target model on the B200. Every verified row is the target's argmax at its position, so the answers are the
target's greedy answers whatever the drafts.
"""
from __future__ import annotations

import time
from typing import Any, Sequence

from .speculation import MAX_DRAFT, NgramIndex, StepPolicy, accept


def context_generate(engine: Any, prompts: Sequence[Sequence[int]], max_new: int | Sequence[int], *,
                     policy: Any = None, collective: Any = None) -> tuple[list[list[int]], dict]:
    """Generate for every prompt (one sequence slot each) with context drafts; returns each request's tokens (up to
    its limit, ending at an end-of-generation token) and step counts."""
    prompts = [list(map(int, p)) for p in prompts]
    limits = [int(max_new)] * len(prompts) if isinstance(max_new, int) else [int(m) for m in max_new]
    if len(prompts) > engine.seqs or len(limits) != len(prompts):
        raise ValueError("one prompt and limit per sequence slot, at most engine.seqs of them")
    for p, limit in zip(prompts, limits):
        if not p or limit < 1 or len(p) + limit > engine.seq_ctx:
            raise ValueError("a prompt needs a token, a positive limit and room in the sequence")
    policy = StepPolicy(engine.max_rows) if policy is None else policy
    for b in range(len(prompts)):
        engine.L.llama_memory_seq_rm(engine.memory, b, -1, -1)
    engine._decode_conf([(t, j, b, False) for b, p in enumerate(prompts) for j, t in enumerate(p[:-1])])
    contexts = [NgramIndex(p) for p in prompts]
    tokens: list[list[int]] = [[] for _ in prompts]
    active = list(range(len(prompts)))
    stats = {"steps": 0, "rows": 0, "drafted": 0, "accepted": 0}
    while active:
        offers = []
        for b in active:
            contexts[b].follow(tokens[b])
            pos = len(prompts[b]) + len(tokens[b]) - 1
            room = min(MAX_DRAFT, limits[b] - len(tokens[b]) - 1, engine.seq_ctx - 1 - pos)
            offer = contexts[b].draft(room) if room > 0 else ([], 0)
            if collective is not None and room > 0 and len(offer[0]) < 2:
                other = collective.draft(contexts[b].tokens, room)
                offer = other if len(other[0]) > len(offer[0]) else offer
            offers.append(offer)
        ks = policy.choose(offers)  # never more drafts than a request offered, nor more rows than the policy's
        rows = []
        for b, (drafts, _), k in zip(active, offers, ks):
            pos = len(prompts[b]) + len(tokens[b]) - 1
            last = tokens[b][-1] if tokens[b] else prompts[b][-1]
            rows += [(t, pos + j, b, True) for j, t in enumerate([last] + list(drafts[:k]))]
        started = time.perf_counter()
        picks = engine._decode_conf(rows)
        policy.observe_step(len(rows), time.perf_counter() - started, any(ks))
        stats["steps"] += 1
        stats["rows"] += len(rows)
        at, done = 0, []
        for b, (drafts, bucket), k in zip(active, offers, ks):
            pos = len(prompts[b]) + len(tokens[b]) - 1
            new = accept(list(drafts[:k]), [tok for tok, _ in picks[at:at + k + 1]])
            at += k + 1
            if k:
                policy.observe_drafts(bucket, k, min(k, len(new) - 1))
                engine.L.llama_memory_seq_rm(engine.memory, b, pos + len(new), -1)  # the rejected positions
            stats["drafted"] += k
            stats["accepted"] += len(new) - 1
            for token in new:
                tokens[b].append(token)
                if engine.eog(token) or len(tokens[b]) >= limits[b]:
                    done.append(b)
                    break
        for b in done:
            if collective is not None:  # this answer becomes a draft source for later requests
                collective.add(tokens[b])
            active.remove(b)
    return tokens, stats
