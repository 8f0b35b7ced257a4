"""ironmule_b200.speculation / draft_model against the reference's own host code.

tests/golden/host_traces.json holds seeded operation sequences run through the reference's
ironmule/speculation.py and ironmule/draft_model.py with every result recorded (made by
tests/golden/make_golden.py); each test replays one family against this package and requires the same
results (floats to 1e-12 relative). The named cases below restate the reference's own unit tests
(tests/engine/test_speculation.py, test_draft_model.py, test_ggml_engine.py)."""
from __future__ import annotations

import json
import math
import random
import time
import types
from pathlib import Path

import pytest

from ironmule_b200 import draft_model as dm
from ironmule_b200 import speculation as sp

TRACES = json.loads((Path(__file__).resolve().parent / "golden" / "host_traces.json").read_text())


def same(a, b) -> bool:
    if isinstance(a, float) or isinstance(b, float):
        if a is None or b is None:
            return a is b
        return math.isclose(float(a), float(b), rel_tol=1e-12, abs_tol=1e-15)
    if isinstance(a, (list, tuple)) and isinstance(b, (list, tuple)):
        return len(a) == len(b) and all(same(x, y) for x, y in zip(a, b))
    if isinstance(a, dict) and isinstance(b, dict):
        return a.keys() == b.keys() and all(same(a[k], b[k]) for k in a)
    return a == b


def test_constants():
    c = TRACES["constants"]
    assert (sp.MAX_DRAFT, sp.MIN_NGRAM, sp.MAX_NGRAM, sp.POLICY_VERSION, sp.MARGIN, sp.COLLECTIVE_BUCKET) == (
        c["MAX_DRAFT"], c["MIN_NGRAM"], c["MAX_NGRAM"], c["POLICY_VERSION"], c["MARGIN"], c["COLLECTIVE_BUCKET"])
    assert (dm.BINS, dm.CHUNK) == (c["BINS"], c["CHUNK"])


def test_draft_matches_reference():
    for case in TRACES["draft"]:
        got = sp.draft(case["context"], case["k"], **case["kw"])
        assert same(list(got), case["result"]), case


def test_ngram_index_matches_reference():
    for trace in TRACES["ngram_index"]:
        index = sp.NgramIndex(trace["prompt"])
        for op, arg, result in trace["ops"]:
            if op == "follow":
                index.follow(arg)
            elif op == "append":
                index.append(arg)
            else:
                got = index.draft(arg)
                assert same([got[0], got[1]], result)


def test_accept_matches_reference():
    for case in TRACES["accept"]:
        assert sp.accept(case["drafts"], case["argmax"]) == case["result"]


@pytest.mark.parametrize("family,cls", [("window_policy", sp.WindowPolicy), ("step_policy", sp.StepPolicy)])
def test_policies_match_reference(family, cls):
    for trace in TRACES[family]:
        policy = cls(trace["rows"])
        for op, args, result in trace["ops"]:
            if op == "choose":
                got = policy.choose([(o[0], o[1]) for o in args[0]])
            else:
                got = getattr(policy, op)(*args)
            assert same(got, result), (op, args, got, result)


def test_collective_index_matches_reference():
    for trace in TRACES["collective"]:
        index = sp.CollectiveIndex(keys=trace["keys"])
        for op, args, result in trace["ops"]:
            if op == "add":
                index.add(*args)
            elif op == "len":
                assert len(index.table) == result
            else:
                got = index.draft(*args)
                assert same([got[0], got[1]], result)


def test_draft_stop_matches_reference():
    for trace in TRACES["draft_stop"]:
        stop = dm.DraftStop()
        for op, args, result in trace["ops"]:
            got = getattr(stop, op)(*args)
            assert same(got, result), (op, args, got, result)


def _sig(tokens):
    return [len(tokens), sum(tokens), *tokens[-8:]]


class _StandIn:
    """The same deterministic stand-in engine the traces were recorded with."""

    def __init__(self, seqs, seed):
        self.seqs, self.memory, self.calls, self.removed = seqs, None, [], []
        self.rng = random.Random(seed)
        self.L = types.SimpleNamespace(llama_memory_seq_rm=self._rm)

    def _rm(self, memory, seq, p0, p1):
        ok = self.rng.random() < 0.9
        self.removed.append([seq, p0, p1, ok])
        return ok

    def _decode_conf(self, rows):
        self.calls.append([list(r) for r in rows])
        return [((token * 7 + pos) % 997, round(self.rng.random(), 4)) for token, pos, _, logits in rows if logits]

    def eog(self, token):
        return token % 97 == 0


class _FixedClock:
    def __init__(self):
        self.now = 0.0

    def __call__(self):
        self.now += 0.004
        return self.now


def test_drafter_matches_reference(monkeypatch):
    monkeypatch.setattr(time, "perf_counter", None)  # replaced per trace below
    for trace in TRACES["drafter"]:
        monkeypatch.setattr(time, "perf_counter", _FixedClock())
        engine = _StandIn(trace["seqs"], trace["seed"])
        drafter = dm.Drafter(engine, max_running=trace["max_running"])
        for op, args, result, state in trace["ops"]:
            if op == "draft":
                wants = {int(k): (v[0], v[1]) for k, v in args[0].items()}
                got = drafter.draft(wants, args[1])
                assert {str(k): v for k, v in got.items()} == result
            elif op == "settle":
                drafter.settle(*args)
            elif op == "release":
                drafter.release(*args)
            assert {str(s): _sig(h) for s, h in drafter.held.items()} == state["held"]
            assert {str(k): v for k, v in drafter.slot_of.items()} == state["slot_of"]
            assert len(engine.calls) == state["calls"]
        assert [[_sig(list(r)) for r in call] for call in engine.calls] == trace["engine_calls"]
        assert engine.removed == trace["engine_removed"]
        summary = {k: v for k, v in drafter.stop.summary().items() if "ms" not in k and "tok_s" not in k}
        assert same(summary, trace["stop_summary"])


def test_suggest_draft_matches_reference():
    for name, want in TRACES["suggest_draft"].items():
        assert dm.suggest_draft(name) == want


# ---- the reference's own unit cases, restated -------------------------------------------------------

def test_a_draft_is_what_followed_the_most_recent_repeat():
    assert sp.draft([5, 6, 7, 8, 1, 5, 6, 7], 3) == ([8, 1, 5], 3)
    assert sp.draft([1, 2, 9, 1, 2, 4, 2], 2) == ([], 0)
    assert sp.draft([1, 2, 9, 1, 2, 4, 2], 2, min_ngram=1) == ([4, 2], 1)
    assert sp.draft([1, 2, 3], 4) == ([], 0) and sp.draft([4, 4], 0) == ([], 0)
    assert sp.accept([3, 4, 5], [3, 4, 9, 7]) == [3, 4, 9] and sp.accept([], [6]) == [6]


def test_plain_and_speculative_steps_are_priced_apart():
    policy = sp.WindowPolicy(rows=8)
    assert policy.plain_price(8) == pytest.approx(1.42)
    policy.observe_step(1, 0.050, False)
    assert policy.plain_price(8) == pytest.approx(0.050 * 1.42)
    assert policy.speculative_price(3, 1) == pytest.approx(0.050 * 1.12)
    policy.observe_step(1, 0.100, False)
    assert policy.plain_price(1) == pytest.approx(0.8 * 0.050 + 0.2 * 0.100)
    for rows, seconds in ((2, 0.080), (4, 0.090), (2, 0.080), (4, 0.090)):
        policy.observe_step(rows, seconds, True)
    assert policy.speculative_price(3, 1) == pytest.approx(0.085)
    assert policy.speculative_price(8, 1) == pytest.approx(0.110)
    out = policy.summary()
    assert out["policy_version"] == 2 and out["speculative_steps"] == 4 and out["plain_steps"] == 2
    assert out["plain_step_ms_by_rows"] == {"1": 60.0} and out["speculative_step_ms_by_rows"]["3"] == 85.0


def test_policy_v3_prices_by_the_median_of_its_recent_steps():
    policy = sp.StepPolicy(rows=8)
    for seconds in (0.010, 0.011, 0.500, 0.012):
        policy.observe_step(2, seconds, False)
    assert policy.price(2) == pytest.approx(0.012)
    for _ in range(40):
        policy.observe_step(2, 0.020, False)
    assert policy.price(2) == pytest.approx(0.020) and len(policy.times[2]) == policy.WINDOW


def test_the_ngram_index_costs_the_new_tokens_not_the_context():
    index = sp.NgramIndex(list(range(5000)) * 4)
    index.draft(7)
    done = index._done
    index.append(1)
    index.draft(7)
    assert index._done == done + 1


def test_randomized_ngram_index_equals_the_scan():
    rng = random.Random(7)
    for _ in range(300):
        vocab = rng.choice([2, 3, 5, 20, 1000])
        prompt = [rng.randrange(vocab) for _ in range(rng.randrange(0, 50))]
        index, answer = sp.NgramIndex(prompt), []
        for _ in range(rng.randrange(1, 40)):
            index.follow(answer)
            k = rng.randrange(0, 9)
            assert index.draft(k) == sp.draft(prompt + answer, k)
            answer += [rng.randrange(vocab) for _ in range(rng.randrange(1, 4))]


def test_sp4_collective_drafts():
    index = sp.CollectiveIndex(keys=1000)
    index.add([5, 6, 7, 8, 9, 10, 11, 12])
    assert index.draft([1, 2, 6, 7, 8, 9], 3) == ([10, 11, 12], sp.COLLECTIVE_BUCKET + 4)
    assert index.draft([1, 2, 3, 8, 9], 2) == ([10, 11], sp.COLLECTIVE_BUCKET + 2)
    index.add([1, 8, 9, 40, 41])
    assert index.draft([0, 8, 9], 2) == ([40, 41], sp.COLLECTIVE_BUCKET + 2)
    small = sp.CollectiveIndex(keys=5)
    small.add(list(range(50)))
    assert len(small.table) == 5


def test_the_drafter_keeps_its_cells_in_step_with_the_text():
    class Engine:
        def __init__(self):
            self.seqs, self.memory, self.calls, self.removed = 2, None, [], []
            self.L = types.SimpleNamespace(llama_memory_seq_rm=lambda m, s, a, b: self.removed.append((s, a, b)) or True)

        def _decode_conf(self, rows):
            self.calls.append(list(rows))
            return [(token + 1, 0.9) for token, _, _, logits in rows if logits]

        def eog(self, token):
            return False

    drafter = dm.Drafter(Engine())
    drafter.stop.by_rows, drafter.stop.call = {1: 0.080, 4: 0.088}, {1: 0.016, 2: 0.018}
    for _ in range(300):
        drafter.stop.learn([0.9, 0.9, 0.9], 3)
        drafter.stop.learn([0.15], 0)
    out = drafter.draft({7: ([10, 11, 12], 4)}, running=1)
    assert out[7] == [13, 14, 15, 16]
    slot = drafter.slot_of[7]
    assert drafter.held[slot] == [10, 11, 12, 13, 14, 15]
    drafter.settle(7, used=4, accepted=1)
    assert drafter.held[slot] == [10, 11, 12, 13] and (slot, 4, -1) in drafter.e.removed
    drafter.draft({7: ([10, 11, 12, 13, 99], 2)}, running=1)
    assert drafter.e.calls[-2][0][:2] == (99, 4)
