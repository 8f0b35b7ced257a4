"""The speculative decoder's slot bookkeeping on the CPU (ironmule_b200.engine.SpecDecoder: start_slots, stop_slot,
finish, the parking of idle slots and the page pool), driven through the decoder's own methods over stand-in models
that record their page-table rows and prefill calls. Invariants checked after every step of random request streams:
an idle slot's rows point only at its private parking pages, outside the pool; a running slot's rows list the pool's
pages for it; two running slots share only full pages the pool indexed (pages whose K/V are final); a request
prefills exactly the prompt tokens the pool did not link (the reference shares prompt prefixes the same way,
ironmule/ggml_engine.py:352-389)."""
import random
import types

import pytest
import torch

from ironmule_b200 import engine
from ironmule_b200.kvpool import PAGE


class StubModel:
    def __init__(self, seqs, pages_per_seq):
        self.max_seqs, self.pages_per_seq = seqs, pages_per_seq
        self.page_table = torch.arange(seqs * pages_per_seq, dtype=torch.int32).view(seqs, -1).clone()
        self.prefills = []

    def prefill_many(self, body):
        self.prefills.append([(item[0], item[1].numel()) + tuple(item[2:]) for item in body])


METHODS = ("_park", "_admit", "_start_shared", "_retire", "stop_slot", "start_slots", "finish", "_check_prompt",
           "request_limit", "start")


def decoder(batch=3, pages_per_seq=16, reserve=4, prefix=True):
    t, d = StubModel(batch, pages_per_seq), StubModel(batch, pages_per_seq)
    dec = types.SimpleNamespace(batch=batch, reserve=reserve, target=t, draft=d, cap=pages_per_seq * PAGE,
                                hist=torch.zeros((batch, pages_per_seq * PAGE), dtype=torch.int32),
                                n=torch.zeros(batch, dtype=torch.int32),
                                target_len=torch.zeros(batch, dtype=torch.int32),
                                stats=torch.zeros((batch, 3), dtype=torch.int64), sampling=None,
                                running=[False] * batch, upto=[0] * batch, end=[0] * batch, reused=[0] * batch,
                                prefill_tokens=0, pool=None)
    for name in METHODS:
        setattr(dec, name, types.MethodType(getattr(engine.SpecDecoder, name), dec))
    if prefix:
        pages = batch * pages_per_seq
        dec.park_base = pages - engine.PARK_PAGES * batch
        dec.pool = engine.PagePool(dec.park_base, batch, pages_per_seq, lead=2)
    for b in range(batch):
        dec._park(b)
    return dec


def check(dec):
    pool = dec.pool
    for b in range(dec.batch):
        for model in (dec.target, dec.draft):
            row = model.page_table[b].tolist()
            if not dec.running[b]:
                park = set(range(dec.park_base + engine.PARK_PAGES * b, dec.park_base + engine.PARK_PAGES * (b + 1)))
                assert set(row) <= park, (b, row)
                assert int(dec.n[b]) == 2 and int(dec.target_len[b]) == 2
            else:
                assert row[:len(pool.seqs[b].pages)] == pool.seqs[b].pages
                assert max(row) < dec.park_base
    owners = {}
    for b in range(dec.batch):
        if dec.running[b]:
            for page in pool.seqs[b].pages:
                owners.setdefault(page, []).append(b)
    for page, slots in owners.items():
        if len(slots) > 1:
            assert page in pool.key_of, (page, slots)


def test_admit_stop_and_park():
    dec = decoder()
    check(dec)
    system = list(range(100, 140))
    p0 = torch.tensor(system + [1, 2, 3], dtype=torch.int32)
    dec.start_slots([(0, p0, 10)])
    check(dec)
    assert dec.target.prefills[-1] == [(0, 42, 0)]
    p1 = torch.tensor(system + [7] * 9, dtype=torch.int32)
    dec.start_slots([(2, p1, 10)])
    check(dec)
    assert dec.reused[2] == 32 and dec.target.prefills[-1] == [(2, 48 - 32, 32)]
    with pytest.raises(ValueError):
        dec.start_slots([(2, p1, 10)])  # a running slot
    with pytest.raises(ValueError):
        dec.start_slots([(1, p1[:1], 10)])  # one prompt token
    dec.n[0] = 43 + 10  # ten tokens generated: 51 final tokens fill a third page
    dec.hist[0, 43:53] = 9
    third = dec.pool.seqs[0].pages[2]
    dec.stop_slot(0)
    check(dec)
    assert not dec.running[0] and list(dec.pool.cached) == [third]
    dec.finish()
    check(dec)
    assert dec.pool.used == 0


@pytest.mark.parametrize("seed", range(5))
def test_random_request_streams(seed):
    rng = random.Random(seed)
    dec = decoder(batch=3, pages_per_seq=12)
    stems = [[rng.randrange(50) for _ in range(90)] for _ in range(2)]
    for _ in range(120):
        idle = [b for b in range(dec.batch) if not dec.running[b]]
        busy = [b for b in range(dec.batch) if dec.running[b]]
        if idle and (not busy or rng.random() < 0.5):
            picks = rng.sample(idle, rng.randint(1, len(idle)))
            items = []
            for b in picks:
                stem = rng.choice(stems)
                ids = stem[:rng.randrange(2, 70)] + [rng.randrange(50) for _ in range(rng.randrange(0, 5))]
                max_new = rng.randrange(1, dec.request_limit() - len(ids) + 1) if len(ids) < dec.request_limit() else 0
                if max_new < 1:
                    continue
                items.append((b, torch.tensor(ids, dtype=torch.int32), max_new))
            if not items:
                continue
            before = [len(p) for p in dec.target.prefills]
            dec.start_slots(items)
            computed = sum(item[1] for call in dec.target.prefills[len(before):] for item in call)
            assert computed == sum(p.numel() - 1 - dec.reused[b] for b, p, _ in items)
        else:
            b = rng.choice(busy)
            grown = rng.randrange(0, int(dec.end[b]) - int(dec.n[b]) + 1)
            n0 = int(dec.n[b])
            dec.hist[b, n0:n0 + grown] = torch.randint(0, 50, (grown,), dtype=torch.int32)
            dec.n[b] = n0 + grown
            dec.stop_slot(b, keep=rng.random() < 0.8)
        check(dec)
    dec.finish(keep=False)
    check(dec)
    assert dec.pool.used == 0


def test_without_a_pool_rows_stay_fixed():
    dec = decoder(prefix=False)
    fixed = dec.target.page_table.clone()
    dec.start_slots([(1, torch.tensor([5, 6, 7, 8], dtype=torch.int32), 3)])
    assert dec.target.prefills[-1] == [(1, 3)]
    dec.stop_slot(1)
    assert torch.equal(dec.target.page_table, fixed)
    assert int(dec.n[1]) == 2 and not dec.running[1]
