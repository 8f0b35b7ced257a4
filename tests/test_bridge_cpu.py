"""The bridge's continuous-batching loop (ironmule_b200.bridge) on the CPU, over a host stand-in decoder whose
slots commit 1 .. k+1 tokens per round from a fixed next-token rule: requests start shortest first in free slots,
`admit` is asked for more while slots are free, tokens are taken one by one with the reference's cancel / eos /
length order (ironmule/ggml_engine.py:1037-1056), a finished request frees its slot at once, results come back in
arrival order with the reference bridge's fields (ironmule_product/ggml_bridge.py:236-291)."""
import random
import types

import pytest
import torch

from ironmule_b200 import bridge


def next_token(ctx):
    return (sum(ctx[-3:]) * 31 + len(ctx)) % 50


def expected(ids, limit, eos=()):
    ctx, out = list(ids), []
    while len(out) < limit:
        t = next_token(ctx)
        ctx.append(t)
        out.append(t)
        if t in eos:
            break
    return out


class FakeDecoder:
    def __init__(self, batch=2, k=3, seed=0, limit=200):
        self.batch, self.k, self.device, self.graph, self.pool = batch, k, "cpu", None, None
        self.running, self.reused = [False] * batch, [0] * batch
        self.ctx, self.end = {}, {}
        self.rng = random.Random(seed)
        self.starts, self.stops, self.captured, self.rounds = [], [], 0, 0
        self.limit = limit
        self.target = types.SimpleNamespace(cfg=types.SimpleNamespace(name="t"))
        self.draft = types.SimpleNamespace(cfg=types.SimpleNamespace(name="d"))

    def request_limit(self):
        return self.limit

    def start_slots(self, items):
        for b, p, max_new in items:
            assert not self.running[b]
            self.running[b] = True
            self.ctx[b] = p.tolist()
            self.end[b] = p.numel() + max_new
            self.starts.append(b)

    def stop_slot(self, b, keep=True):
        assert self.running[b]
        self.running[b] = False
        self.stops.append(b)

    def finish(self, keep=True):
        for b in range(self.batch):
            if self.running[b]:
                self.stop_slot(b, keep)

    def capture(self):
        self.graph = object()
        self.captured += 1

    def step(self):
        self.rounds += 1
        out = {}
        for b in range(self.batch):
            if not self.running[b]:
                continue
            new = []
            for _ in range(self.rng.randint(1, self.k + 1)):
                if len(self.ctx[b]) >= self.end[b]:
                    break
                t = next_token(self.ctx[b])
                self.ctx[b].append(t)
                new.append(t)
            if new:
                out[b] = new
        return out


class Tok:
    def decode(self, ids):
        return " ".join(map(str, ids))


def prompts(n, seed=1):
    rng = random.Random(seed)
    return [[rng.randrange(50) for _ in range(rng.randrange(2, 30))] for _ in range(n)]


def test_generate_many_serves_more_requests_than_slots():
    dec = FakeDecoder(batch=2)
    br = bridge.DeviceBridge(dec, Tok())
    ps = prompts(5)
    limits = [7, 3, 12, 1, 9]
    seen = {i: [] for i in range(5)}
    res = br.generate_many(ps, limits, on_tokens=[seen[i].append for i in range(5)])
    for i, r in enumerate(res):
        want = expected(ps[i], limits[i])
        assert r.tokens == want and seen[i] == want and r.token_count == len(want)
        assert r.finish_reason == "length" and r.text == " ".join(map(str, want))
    assert len(dec.starts) == 5 and sorted(dec.stops) == sorted(dec.starts) and dec.captured == 1
    assert br.free_slots() == 2 and br.counters()["requests"] == 5


def test_shortest_prompt_first_and_slot_reuse():
    dec = FakeDecoder(batch=1)
    ps = [[1] * 20, [2] * 3, [3] * 9]
    order = []
    jobs = [bridge.Job(p, 2, emit=lambda t, i=i: order.append(i)) for i, p in enumerate(ps)]
    served = bridge.serve(dec, jobs)
    assert served == jobs and [j.reason for j in jobs] == ["length"] * 3
    assert order == [1, 1, 2, 2, 0, 0] and dec.starts == [0, 0, 0]


def test_eos_ends_a_request_and_is_kept_out_of_the_text():
    ps = prompts(3, seed=4)
    full = expected(ps[0], 20)
    eos = full[4]
    dec = FakeDecoder(batch=2)
    res = bridge.DeviceBridge(dec, Tok(), eos_ids=[eos]).generate_many(ps, 20)
    for i, r in enumerate(res):
        want = expected(ps[i], 20, eos=(eos,))
        assert r.tokens == want
        assert r.finish_reason == ("stop" if want[-1] == eos else "length")
        assert r.text == " ".join(str(t) for t in want if t != eos)
    assert res[0].finish_reason == "stop" and len(res[0].tokens) <= 5


def test_admit_hands_over_requests_while_slots_are_free():
    dec = FakeDecoder(batch=2)
    extra = prompts(4, seed=7)
    calls = []

    def admit(free):
        calls.append(free)
        take, extra[:] = extra[:free], extra[free:]
        return [(ids, 5, None) for ids in take]

    ps = prompts(1, seed=3)
    res = bridge.DeviceBridge(dec).generate_many(ps, 5, admit=admit)
    assert len(res) == 5 and all(r.finish_reason == "length" and r.token_count == 5 for r in res)
    assert calls[0] == 2 and not extra
    with pytest.raises(ValueError):
        bridge.DeviceBridge(FakeDecoder()).generate_many(ps, 5, admit=lambda free: [(ps[0], 5, None, [3])])


def test_cancel_before_and_during_a_request():
    dec = FakeDecoder(batch=1)
    got = []
    ps = prompts(3, seed=9)
    never = bridge.Job(ps[0], 10, cancelled=lambda: True)
    during = bridge.Job(ps[1], 30, emit=got.append, cancelled=lambda: len(got) >= 4)
    normal = bridge.Job(ps[2], 6)
    bridge.serve(dec, [never, during, normal])
    assert never.reason == "cancelled" and never.tokens == []
    assert during.reason == "cancelled" and during.tokens == expected(ps[1], 4)
    assert normal.reason == "length" and normal.tokens == expected(ps[2], 6)
    assert len(dec.starts) == 2


def test_refusals():
    br = bridge.DeviceBridge(FakeDecoder(limit=40))
    with pytest.raises(ValueError):
        br.generate_many([[1, 2, 3]], 4, boundaries=[[1]])
    with pytest.raises(ValueError):
        br.generate([5], 4)
    with pytest.raises(ValueError):
        br.generate([1] * 30, 11)
    r = br.generate([1] * 30, 10)
    assert r.token_count == 10 and r.metadata["configuration"] == "b200"


def test_serve_passes_device_prompts():
    dec = FakeDecoder(batch=1)
    seen = []
    real = dec.start_slots

    def spy(items):
        seen.extend(p for _, p, _ in items)
        real(items)

    dec.start_slots = spy
    bridge.serve(dec, [bridge.Job([4, 5, 6], 2)])
    assert seen[0].dtype == torch.int32 and seen[0].tolist() == [4, 5, 6]


def test_an_invalid_admitted_request_ends_alone():
    """A request admitted while others run that cannot be served (one prompt token, or too long) ends at once with
    an error; the running requests finish normally."""
    dec = FakeDecoder(batch=2, limit=60)
    ps = prompts(2, seed=11)
    handed = []

    def admit(free):
        if handed:
            return []
        handed.append(free)
        return [([7], 4, None), ([1] * 50, 20, None)]

    res = bridge.DeviceBridge(dec).generate_many(ps, 6, admit=admit)
    assert [r.finish_reason for r in res] == ["length", "length", "error", "error"]
    assert res[2].token_count == 0 and "two prompt tokens" in res[2].metadata["error"]
    assert "do not fit" in res[3].metadata["error"]
    assert res[0].tokens == expected(ps[0], 6) and res[1].tokens == expected(ps[1], 6)
    assert not any(dec.running)


def test_an_exception_while_serving_stops_the_running_slots():
    dec = FakeDecoder(batch=2)
    ps = prompts(2, seed=12)

    def boom(token):
        raise RuntimeError("the client went away")

    with pytest.raises(RuntimeError):
        bridge.serve(dec, [bridge.Job(ps[0], 20, emit=boom), bridge.Job(ps[1], 20)])
    assert not any(dec.running) and sorted(dec.stops) == [0, 1]
