"""Host logic of the device draft engine (ironmule_b200.engine): the decode plan that packs llama.cpp-style rows
of several sequences into forwards, and the engine's position bookkeeping for `llama_memory_seq_rm` (the calls the
reference's Drafter makes, ironmule/draft_model.py:194-270). No device work: the checks here raise before any
launch."""
import random
import types

import pytest

from ironmule_b200 import engine


def check_plan(wants, step, budget, logit_budget):
    plan = engine.decode_plan(wants, step, budget, logit_budget)
    seen = [0] * len(wants)
    for chunks, logit_rows in plan:
        assert chunks and sum(n for _, _, n in chunks) <= budget
        assert len({i for i, _, _ in chunks}) == len(chunks)  # one chunk per sequence per forward
        assert 0 <= logit_rows <= logit_budget
        row = 0
        last_logit = -1
        for i, off, n in chunks:
            assert 1 <= n <= step and off == seen[i]
            for j in range(n):
                if wants[i][off + j]:
                    last_logit = row + j
            seen[i] += n
            row += n
        assert logit_rows == last_logit + 1  # exactly the rows up to the last one that needs logits
    assert seen == [len(w) for w in wants]
    return plan


def test_plan_puts_logit_chunks_first():
    plan = check_plan([[False] * 40 + [True], [True], [False, False, True]], 32, 64, 32)
    assert plan == [([(1, 0, 1), (2, 0, 3), (0, 0, 32)], 4), ([(0, 32, 9)], 9)]


def test_plan_respects_the_logit_budget():
    wants = [[True] * 10 for _ in range(5)]
    plan = check_plan(wants, 32, 320, 32)
    assert [lr for _, lr in plan] == [30, 20]


def test_plan_refuses_bad_limits():
    with pytest.raises(ValueError):
        engine.decode_plan([[True]], 32, 16, 32)
    with pytest.raises(ValueError):
        engine.decode_plan([[True]], 32, 64, 8)


@pytest.mark.parametrize("seed", range(8))
def test_plan_randomized(seed):
    rng = random.Random(seed)
    wants = [[rng.random() < 0.2 for _ in range(rng.randrange(0, 90))] for _ in range(rng.randrange(1, 9))]
    step = rng.choice([1, 8, 32])
    check_plan(wants, step, rng.choice([step, 64, 320]), rng.choice([step, 32]))


def stub_engine(seqs=2, ctx=64):
    model = types.SimpleNamespace(max_rows=32, max_logit_rows=32, max_seqs=seqs, max_ctx=ctx)
    return engine.DeviceDraftEngine(model, eog_ids=[5])


def test_seq_rm_bookkeeping():
    e = stub_engine()
    e.filled = [20, 7]
    assert e.L.llama_memory_seq_rm(None, 0, 12, -1) and e.filled[0] == 12
    assert not e.L.llama_memory_seq_rm(None, 0, 3, 6)  # a hole below kept positions
    assert e.L.llama_memory_seq_rm(None, 0, 6, 40) and e.filled[0] == 6  # reaches past the end: a tail
    assert e.L.llama_memory_seq_rm(None, 1, -1, -1) and e.filled == [6, 0]
    with pytest.raises(ValueError):
        e.L.llama_memory_seq_rm(None, 2, 0, -1)
    assert e.eog(5) and not e.eog(6) and e.seqs == 2 and e.memory is None


def test_rows_must_continue_each_sequence():
    e = stub_engine()
    e.filled = [3, 0]
    with pytest.raises(ValueError, match="expected 3"):
        e._decode_conf([(1, 4, 0, True)])
    with pytest.raises(ValueError, match="expected 1"):
        e._decode_conf([(1, 0, 1, False), (2, 2, 1, True)])
    with pytest.raises(ValueError):
        e._decode_conf([(1, 0, 2, True)])
    with pytest.raises(ValueError, match="positions"):
        e._decode_conf([(1, 3 + j, 0, False) for j in range(62)])
    assert e._decode_conf([]) == [] and e.filled == [3, 0]


def test_the_draft_model_needs_a_logit_block_per_chunk():
    model = types.SimpleNamespace(max_rows=32, max_logit_rows=8, max_seqs=1, max_ctx=64)
    with pytest.raises(ValueError):
        engine.DeviceDraftEngine(model)
