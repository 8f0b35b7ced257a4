"""The shared-prefix page pool (ironmule_b200/kvpool.py) on the CPU: sharing of full prompt pages, reference
counts, least-recently-used eviction of cached pages, refusal without side effects, and a randomized run that
models what each page's K/V holds and checks that a shared page always holds the sharer's own token chain and that
no write ever lands in a page another sequence holds or the index lists (the properties the reference's pool keeps
for its cells, ironmule/ggml_engine.py:280-432)."""
import random

import pytest

from ironmule_b200.kvpool import PAGE, PagePool


def toks(n, base=0):
    return [base + i for i in range(n)]


def test_place_fresh_pages_and_row():
    pool = PagePool(pages=8, slots=2, row_pages=4)
    slot, keep = pool.place(toks(40), 10)
    assert (slot, keep) == (0, 0)
    row = pool.row(0)
    assert len(row) == 4 and len(set(row)) == 4  # 50 tokens -> 4 distinct pages
    assert pool.row(0, 6)[4:] == [row[-1], row[-1]]
    with pytest.raises(ValueError):
        pool.row(0, 3)
    assert pool.used == 4 and len(pool.free) == 4


def test_share_full_pages_after_release():
    pool = PagePool(pages=16, slots=2, row_pages=8)
    a = toks(48)
    pool.place(a, 0)
    pool.commit(0, a)
    pages_a = pool.row(0)[:3]
    pool.release(0)
    assert pool.used == 0 and len(pool.cached) == 3
    b = a[:40] + [999] * 10
    slot, keep = pool.place(b, 5)
    assert keep == 32 and pool.row(slot)[:2] == pages_a[:2]
    assert pool.row(slot)[2] != pages_a[2]
    assert pool.shared_tokens == 32


@pytest.mark.parametrize("lead,length,expect", [(1, 48, 32), (2, 48, 32), (1, 49, 48), (2, 49, 32), (2, 50, 48)])
def test_lead_tokens_always_computed(lead, length, expect):
    pool = PagePool(pages=16, slots=2, row_pages=8, lead=lead)
    a = toks(64)
    pool.place(a, 0)
    pool.commit(0, a)
    pool.release(0)
    _, keep = pool.place(a[:length], 4)
    assert keep == expect and keep <= length - lead


def test_running_sequences_share_with_refcounts():
    pool = PagePool(pages=16, slots=3, row_pages=8)
    a = toks(40)
    pool.place(a, 8)
    pool.commit(0, a[:32])  # two full pages now final
    _, keep = pool.place(a[:35] + [7, 7], 3)
    assert keep == 32
    shared = pool.row(0)[:2]
    assert pool.row(1)[:2] == shared
    assert all(pool.ref[p] == 2 for p in shared)
    pool.release(0)
    assert all(pool.ref[p] == 1 for p in shared)  # still held by slot 1
    pool.release(1)
    assert pool.used == 0 and set(shared) <= set(pool.cached)


def test_eviction_lru_deepest_first():
    pool = PagePool(pages=6, slots=1, row_pages=6)
    a = toks(48)
    pool.place(a, 0)
    pool.commit(0, a)
    pa = pool.row(0)[:3]
    pool.release(0)
    b = toks(32, base=1000)
    pool.place(b, 0)
    pool.commit(0, b)
    pb = pool.row(0)[:2]
    pool.release(0)
    assert list(pool.cached) == [pa[2], pa[1], pa[0], pb[1], pb[0]]
    # a new unrelated request of 4 pages takes the free page, then evicts a's chain from its end
    pool.place(toks(64, base=5000), 0)
    assert list(pool.cached) == [pb[1], pb[0]]
    pool.release(0, keep=False)
    # b is still cached whole; a is gone
    assert pool.longest(b) == pb and pool.longest(a) == []


def test_eviction_keeps_the_shorter_prefix_reachable():
    pool = PagePool(pages=4, slots=1, row_pages=4)
    a = toks(48)
    pool.place(a, 0)
    pool.commit(0, a)
    pool.release(0)
    pool.place(toks(20, base=500), 0)  # needs 2 pages: the free one and a's deepest
    pool.release(0, keep=False)
    assert len(pool.longest(a)) == 2


def test_refusal_changes_nothing():
    pool = PagePool(pages=4, slots=2, row_pages=4)
    pool.place(toks(40), 8)  # 3 pages
    before = pool.summary(), dict(pool.ref), list(pool.free)
    assert pool.place(toks(40, base=100), 8) is None
    assert (pool.summary(), dict(pool.ref), list(pool.free)) == before
    pool.place(toks(10, base=100), 0, slot=1)
    assert pool.place(toks(4), 0) is None  # no free slot


def test_release_without_keep_drops_index():
    pool = PagePool(pages=8, slots=1, row_pages=8)
    a = toks(32)
    pool.place(a, 0)
    pool.commit(0, a)
    pool.release(0, keep=False)
    assert pool.index == {} and pool.key_of == {} and len(pool.free) == 8
    assert pool.place(a, 0)[1] == 0


def test_errors():
    pool = PagePool(pages=8, slots=2, row_pages=2)
    with pytest.raises(ValueError):
        PagePool(0, 1, 1)
    with pytest.raises(ValueError):
        pool.place([], 3)
    with pytest.raises(ValueError):
        pool.place(toks(30), 3)  # 33 tokens > 2 pages
    pool.place(toks(20), 4, slot=1)
    with pytest.raises(ValueError):
        pool.place(toks(5), 1, slot=1)
    with pytest.raises(ValueError):
        pool.commit(1, toks(33))
    pool.commit(1, toks(16))
    with pytest.raises(ValueError):
        pool.commit(1, toks(16, base=3))  # contradicts the indexed page
    with pytest.raises(ValueError):
        pool.commit(1, toks(10))  # shorter than the indexed pages


def _check_accounting(pool):
    held, cached, free = set(pool.ref), set(pool.cached), set(pool.free)
    assert not (held & cached) and not (held & free) and not (cached & free)
    assert held | cached | free == set(range(pool.pages))
    assert len(pool.free) == len(free)
    assert set(pool.key_of) == set(pool.index.values()) and cached <= set(pool.key_of)
    assert set(pool.node_of) == set(pool.key_of) and all(pool.index[k] == p for p, k in pool.key_of.items())
    assert len(set(pool.node_of.values())) == len(pool.node_of)
    counts = {}
    for seq in pool.seqs.values():
        for p in seq.pages:
            counts[p] = counts.get(p, 0) + 1
    assert counts == pool.ref


@pytest.mark.parametrize("seed", range(6))
def test_randomized_page_contents(seed):
    rng = random.Random(seed)
    lead = rng.choice([1, 2])
    pool = PagePool(pages=rng.choice([12, 20, 40]), slots=3, row_pages=6, lead=lead)
    content = {}  # page -> {slot in page: the token chain through that position}
    stems = [[rng.randrange(5) for _ in range(60)] for _ in range(3)]
    running = {}  # slot -> (its token stream, tokens written so far)

    def write(slot, upto):
        stream, done = running[slot]
        pages = pool.seqs[slot].pages
        for pos in range(done, upto):
            page = pages[pos // PAGE]
            # never write a page another sequence holds or the index lists
            assert pool.ref[page] == 1 and page not in pool.key_of
            content.setdefault(page, {})[pos % PAGE] = tuple(stream[:pos + 1])
        running[slot] = (stream, upto)

    for _ in range(300):
        op = rng.random()
        free_slots = [s for s in range(pool.slots) if s not in pool.seqs]
        if free_slots and op < 0.45:
            stem = rng.choice(stems)
            cut = rng.randrange(2, 60)
            prompt = stem[:cut] + [rng.randrange(5) for _ in range(rng.randrange(0, 8))]
            limit = rng.randrange(0, 24)
            stream = prompt + [rng.randrange(5) for _ in range(limit)]
            placed = pool.place(prompt, limit, slot=rng.choice(free_slots))
            if placed is None:
                continue
            slot, keep = placed
            assert keep % PAGE == 0 and keep <= len(prompt) - lead
            # every shared page holds exactly this prompt's chain at every position
            for pos in range(keep):
                assert content[pool.seqs[slot].pages[pos // PAGE]][pos % PAGE] == tuple(prompt[:pos + 1])
            running[slot] = (stream, keep)
            write(slot, len(prompt) - lead)
            pool.commit(slot, prompt[:len(prompt) - lead])
        elif pool.seqs and op < 0.8:
            slot = rng.choice(list(pool.seqs))
            stream, done = running[slot]
            upto = min(len(stream), done + rng.randrange(1, 12))
            write(slot, upto)
            pool.commit(slot, stream[:upto])
        elif pool.seqs:
            slot = rng.choice(list(pool.seqs))
            pool.release(slot, keep=rng.random() < 0.8)
            del running[slot]
        _check_accounting(pool)
    assert pool.shared_tokens > 0


def test_a_child_under_a_dropped_parent_is_never_matched():
    pool = PagePool(pages=8, slots=2, row_pages=4)
    x, y, w = toks(16, 100), toks(16, 200), toks(16, 300)
    pool.place(x + y + [1], 0, slot=0)
    pool.commit(0, x + y)
    a0, a1 = pool.row(0)[:2]
    _, keep = pool.place(x + [5, 6], 0, slot=1)
    assert keep == 16 and pool.row(1)[0] == a0
    pool.release(0)  # a1 cached; a0 still held by slot 1
    pool.release(1, keep=False)  # a0 unindexed and freed; a1 stays cached under a0's old node
    assert a1 in pool.cached and a0 in pool.free
    pool.place(w + y + [2], 0, slot=0)  # reuses a0's id for another chain
    pool.commit(0, w + y)
    assert pool.row(0)[0] == a0 and pool.longest(w + y) == pool.row(0)[:2]
    assert pool.row(0)[1] != a1 or a1 not in pool.cached


def test_a_chain_whose_canonical_page_was_dropped_is_reindexed():
    pool = PagePool(pages=12, slots=2, row_pages=4)
    x, y = toks(16, 10), toks(16, 40)
    pool.place(x + [0], 0, slot=0)
    pool.place(x + y + [0], 0, slot=1)  # computed apart: nothing was indexed yet
    pool.commit(0, x)
    pool.commit(1, x + y)  # x is slot 0's page; slot 1's second page goes under it
    b0, b1 = pool.row(1)[:2]
    assert pool.longest(x + y) == [pool.row(0)[0], b1]
    pool.release(0, keep=False)  # the canonical x page goes
    assert pool.longest(x + y) == []
    pool.commit(1, x + y + toks(3))
    assert pool.longest(x + y) == [b0, b1]
