"""Prompt-prefix sharing through the page pool on the device (SpecDecoder(prefix_cache=True)): sequences of a
batch that share a system prompt, and a later turn that extends an earlier request's prompt and answer, link the
shared full pages instead of computing them. A position's K/V depend only on the tokens up to it and every kernel
is row-invariant, so the caches hold the same bits as a full prefill and the answers equal plain greedy decoding
(the reference shares prompt prefixes the same way, ironmule/ggml_engine.py:352-389)."""
from __future__ import annotations

import pytest
import torch

from ironmule_b200 import engine

pytestmark = pytest.mark.gpu


def tiny(name, seed, b, rows=32):
    return engine.QuantModel(engine.PRESETS[name], "cuda", seed=seed, sigma=0.08, max_ctx=256, max_seqs=b,
                             max_rows=rows, max_logit_rows=rows)


def slots(model, b, n):
    """Slot b's first n positions of both caches through its page-table row: [layers, n, Hkv, D] each."""
    pages = model.page_table[b].long()
    out = []
    for cache in (model.k_cache, model.v_cache):
        t = cache[:, pages].permute(0, 1, 3, 2, 4)
        out.append(t.reshape(model.cfg.layers, -1, model.cfg.kv_heads, model.cfg.head_dim)[:, :n])
    return out


def test_batch_sharing_a_system_prompt(cuda):
    b = 3
    target, draft = tiny("tiny-target", 1, b), tiny("tiny-draft", 2, b)
    gen = torch.Generator().manual_seed(21)
    system = torch.randint(0, 1000, (40,), generator=gen)
    prompts = [torch.cat([system, torch.randint(0, 1000, (n,), generator=gen)]).to(torch.int32) for n in (7, 12, 3)]
    dec = engine.SpecDecoder(target, draft, k=4, batch=b, prefix_cache=True)
    dec.start([p.to(cuda) for p in prompts], max_new=24)
    # the first prompt computes the system prompt; the others link its two full pages (wave two)
    assert dec.pool.shared_tokens == 64
    assert dec.prefill_tokens == sum(p.numel() - 1 for p in prompts) - 64
    rows = [dec.pool.row(s) for s in range(b)]
    assert rows[1][:2] == rows[0][:2] == rows[2][:2] and len(set(rows[1][2:4]) | set(rows[0][2:4])) == 4
    # the caches hold the bits a full prefill writes
    ref_t, ref_d = tiny("tiny-target", 1, b), tiny("tiny-draft", 2, b)
    body = [(s, p[:-1].to(cuda)) for s, p in enumerate(prompts)]
    ref_t.prefill_many(body)
    ref_d.prefill_many(body)
    torch.cuda.synchronize()
    for s, p in enumerate(prompts):
        for mine, ref in ((target, ref_t), (draft, ref_d)):
            for x, y in zip(slots(mine, s, p.numel() - 1), slots(ref, s, p.numel() - 1)):
                assert torch.equal(x.view(torch.int16), y.view(torch.int16)), s
    while not dec.done():
        dec.run_rounds(3)
    solo = tiny("tiny-target", 1, 1)
    for s, p in enumerate(prompts):
        assert dec.generated(s, p.numel()) == engine.greedy_decode(solo, p.to(cuda), 24), s


def test_next_turn_shares_prompt_and_answer(cuda):
    """Turn two's prompt is turn one's prompt + answer + a new message: the pages of turn one's committed tokens
    (kept as a cache when the slot is released) are linked, and the round runs as a captured graph whose page
    tables were rewritten in place."""
    b = 2
    target, draft = tiny("tiny-target", 1, b), tiny("tiny-draft", 2, b)
    gen = torch.Generator().manual_seed(33)
    first = [torch.randint(0, 1000, (n,), generator=gen).to(torch.int32).tolist() for n in (30, 50)]
    dec = engine.SpecDecoder(target, draft, k=4, batch=b, prefix_cache=True)
    dec.start([torch.tensor(p, dtype=torch.int32, device=cuda) for p in first], max_new=20)
    dec.round()
    dec.capture()
    out1 = dec.generate(first, max_new=20)  # re-places the same prompts: their prompt pages are linked
    assert dec.pool.shared_tokens == 16 + 48
    second = [p + o + torch.randint(0, 1000, (5,), generator=gen).tolist() for p, o in zip(first, out1)]
    before = dec.pool.shared_tokens
    out2 = dec.generate(second, max_new=20)
    assert dec.pool.shared_tokens - before >= (30 + 18) // 16 * 16 + (50 + 18) // 16 * 16
    solo = tiny("tiny-target", 1, 1)
    for s in range(b):
        assert out1[s] == engine.greedy_decode(solo, torch.tensor(first[s], device=cuda), 20), s
        assert out2[s] == engine.greedy_decode(solo, torch.tensor(second[s], device=cuda), 20), s
    dec.finish(keep=False)
    assert dec.pool.used == 0 and len(dec.pool.free) + len(dec.pool.cached) == dec.pool.pages


def test_tree_decoder_with_shared_prefix(cuda):
    """Tree speculation moves accepted nodes' K/V through the page table (im_tree_compact): with pooled pages
    the answers still equal plain greedy decoding."""
    b = 2
    target, draft = tiny("tiny-target", 1, b, 32 * b), tiny("tiny-draft", 2, b, 32 * b)
    gen = torch.Generator().manual_seed(44)
    system = torch.randint(0, 1000, (35,), generator=gen)
    prompts = [torch.cat([system, torch.randint(0, 1000, (n,), generator=gen)]).to(torch.int32) for n in (4, 9)]
    dec = engine.TreeDecoder(target, draft, branch=(4, 2, 2), batch=b, prefix_cache=True)
    dec.start([p.to(cuda) for p in prompts], max_new=30)
    assert dec.pool.shared_tokens == 32
    dec.round()
    dec.capture()
    while not dec.done():
        dec.run_rounds(2)
    solo = tiny("tiny-target", 1, 1)
    for s, p in enumerate(prompts):
        assert dec.generated(s, p.numel()) == engine.greedy_decode(solo, p.to(cuda), 30), s
