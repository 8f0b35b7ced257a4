"""Context speculation's step loop (ironmule_b200.context_spec, the reference's ggml step without a draft model,
ironmule/ggml_engine.py:1155-1343) on the CPU over a stand-in engine whose "target" is a fixed next-token rule and
which enforces the device engine's contract (rows continue each sequence from its first free position; tail
removal only). The answers must equal greedy decoding under that rule whatever the policy drafts; on periodic text
the n-gram drafts are accepted and the steps shrink; the policy sees every step and every draft outcome; the
collective index receives finished answers."""
import types

import pytest

from ironmule_b200 import context_spec
from ironmule_b200.speculation import CollectiveIndex, StepPolicy


def rule_periodic(ctx):
    return ctx[-5] if len(ctx) >= 5 else (ctx[-1] + 1) % 50  # period-5 continuation


def rule_mixed(ctx):
    return (sum(ctx[-3:]) * 7 + len(ctx)) % 50


class StandIn:
    def __init__(self, rule, seqs=4, seq_ctx=400, max_rows=32, eog=()):
        self.rule, self.seqs, self.seq_ctx, self.max_rows, self.memory = rule, seqs, seq_ctx, max_rows, None
        self.hist = {b: [] for b in range(seqs)}
        self.eog_ids = set(eog)
        self.calls = []
        self.L = types.SimpleNamespace(llama_memory_seq_rm=self._rm)

    def _rm(self, memory, seq, p0, p1):
        assert p1 == -1
        del self.hist[seq][max(p0, 0):]
        return True

    def eog(self, token):
        return token in self.eog_ids

    def _decode_conf(self, rows):
        self.calls.append(len(rows))
        out = []
        for token, pos, seq, logits in rows:
            assert pos == len(self.hist[seq]), "rows must continue the sequence"
            self.hist[seq].append(token)
            if logits:
                out.append((self.rule(self.hist[seq]), 0.5))
        return out


def greedy(rule, prompt, n, eog=()):
    ctx, out = list(prompt), []
    while len(out) < n:
        t = rule(ctx)
        ctx.append(t)
        out.append(t)
        if t in eog:
            break
    return out


@pytest.mark.parametrize("rule", [rule_periodic, rule_mixed])
def test_answers_equal_greedy(rule):
    prompts = [[3, 9, 4, 1, 7, 3, 9, 4, 1, 7, 3], [5, 5], [1], list(range(20))]
    limits = [40, 25, 30, 12]
    eng = StandIn(rule)
    tokens, stats = context_spec.context_generate(eng, prompts, limits)
    assert tokens == [greedy(rule, p, n) for p, n in zip(prompts, limits)]
    assert stats["rows"] == sum(eng.calls[1:])  # the first call is the prefill


def test_periodic_text_accepts_drafts():
    prompt = [3, 9, 4, 1, 7] * 3
    policy = StepPolicy(32)
    eng = StandIn(rule_periodic)
    tokens, stats = context_spec.context_generate(eng, [prompt], 60, policy=policy)
    assert tokens[0] == greedy(rule_periodic, prompt, 60)
    assert stats["accepted"] > 20 and stats["steps"] < 40
    assert stats["steps"] + stats["accepted"] == 60
    assert policy.drafted == stats["drafted"] and policy.accepted == stats["accepted"]


def test_end_token_and_collective():
    prompt = [2, 8, 6]
    full = greedy(rule_mixed, prompt, 30)
    eos = full[9]
    col = CollectiveIndex()
    eng = StandIn(rule_mixed, eog=[eos])
    tokens, _ = context_spec.context_generate(eng, [prompt, prompt + [1]], 30, collective=col)
    assert tokens[0] == greedy(rule_mixed, prompt, 30, eog=(eos,)) and tokens[0][-1] == eos
    assert col.added == 2


def test_refusals():
    eng = StandIn(rule_mixed, seqs=2, seq_ctx=50)
    with pytest.raises(ValueError):
        context_spec.context_generate(eng, [[1], [2], [3]], 5)
    with pytest.raises(ValueError):
        context_spec.context_generate(eng, [[1] * 45], 10)
    with pytest.raises(ValueError):
        context_spec.context_generate(eng, [[]], 3)
