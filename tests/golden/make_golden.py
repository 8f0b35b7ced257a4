"""Generates the committed golden fixtures in tests/golden/ from the reference itself.

Run where the reference tree is checked out ($IRONMULE_REFERENCE, else a directory named "reference" beside
this repository):

    python tests/golden/make_golden.py

1. qmv_*.npz -- inputs and outputs of the reference's own Metal qmv kernels (IronMule
   ironmule/qmv_k3840.py, qmv_shared.py, qmv_fast_shared.py, qmv_variant.py), compiled for the CPU by
   oracle/build_ref.py. Each file holds seeded weights quantised by oracle/quant.py, bf16 activations and
   the kernel's bf16 outputs under both `bfloat + bfloat` semantics (`y_bf0`, `y_bf1`).
2. host_traces.json -- the reference's own pure-Python host code (ironmule/speculation.py,
   ironmule/draft_model.py) driven through seeded random operation sequences, every call's result
   recorded. The reference package's __init__ imports MLX, so the two modules are loaded through a
   throwaway stub package whose __path__ points at the reference's ironmule/ directory.

Nothing at test time reads the reference: the tests replay these files against ironmule_b200.
"""
from __future__ import annotations

import json
import os
import random
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
REF = Path(os.environ.get("IRONMULE_REFERENCE", REPO.parent / "reference"))
sys.path.insert(0, str(REPO))

QMV_CASES = [
    # (kernel, K, N, M, vpt, seed)
    ("qmv_port", 320, 24, 2, 8, 1),          # runtime K with a partial tail block
    ("qmv_port", 1088, 40, 3, 8, 2),         # 4.25 blocks
    ("qmv_k3840", 3840, 48, 3, 8, 3),
    ("qmv_variant", 3840, 64, 2, 8, 4),
    ("qmv_shared_x1", 3840, 16, 1, 8, 5),
    ("qmv_shared_x2", 3840, 16, 2, 8, 6),
    ("qmv_fast_k4096_x1", 4096, 16, 1, 16, 7),
    ("qmv_fast_k4096_x2", 4096, 16, 2, 16, 8),
    ("qmv_fast_k15360_x2", 15360, 8, 2, 16, 9),
]


def make_qmv() -> None:
    sys.path.insert(0, str(REPO / "oracle"))
    from oracle import bf16, build_ref, qmv, quant

    build_ref.build()
    for name, k, n, m, vpt, seed in QMV_CASES:
        rng = np.random.default_rng(seed)
        w = rng.normal(0.0, 0.02, (n, k)).astype(np.float32)
        wq, s, b = quant.quantize(w)
        x = bf16.from_f32(rng.normal(0.0, 1.0, (m, k)).astype(np.float32))
        y0 = qmv.emu(name, wq, s, b, x, False)
        y1 = qmv.emu(name, wq, s, b, x, True)
        np.savez_compressed(HERE / f"qmv_{name}_k{k}.npz", wq=wq, scales=s, biases=b, x=x, y_bf0=y0, y_bf1=y1,
                            vpt=np.int32(vpt))
        print(f"qmv_{name}_k{k}.npz", y0.shape)


def _load_reference_host():
    stub = Path(tempfile.mkdtemp(prefix="imshim_")) / "ironmule"
    stub.mkdir()
    (stub / "__init__.py").write_text(f"__path__ = [{str(REF / 'ironmule')!r}]\n")
    sys.path.insert(0, str(stub.parent))
    import ironmule.draft_model as dm  # noqa: PLC0415
    import ironmule.speculation as sp  # noqa: PLC0415
    return sp, dm


def _draft_cases(sp, rng: random.Random) -> list:
    out = []
    for _ in range(400):
        vocab = rng.choice([2, 3, 5, 20, 1000])
        ctx = [rng.randrange(vocab) for _ in range(rng.randrange(0, 60))]
        k = rng.randrange(0, 9)
        kw = {}
        if rng.random() < 0.25:
            kw["min_ngram"] = rng.choice([1, 2])
            kw["max_ngram"] = rng.choice([2, 3, 4])
        out.append({"context": ctx, "k": k, "kw": kw, "result": list(map(list_or, sp.draft(ctx, k, **kw)))})
    return out


def list_or(v):
    return list(v) if isinstance(v, (list, tuple)) else v


def _ngram_cases(sp, rng: random.Random) -> list:
    """Incremental index traces: (op, arg, result)."""
    traces = []
    for _ in range(150):
        vocab = rng.choice([2, 3, 5, 20, 1000])
        prompt = [rng.randrange(vocab) for _ in range(rng.randrange(0, 50))]
        index, answer, ops = sp.NgramIndex(prompt), [], []
        for _ in range(rng.randrange(1, 30)):
            if rng.random() < 0.5:
                index.follow(answer)
                ops.append(["follow", list(answer), None])
            else:
                for token in answer[len(index.tokens) - len(prompt):]:
                    index.append(token)
                    ops.append(["append", token, None])
            k = rng.randrange(0, 9)
            res = index.draft(k)
            ops.append(["draft", k, [list(res[0]), res[1]]])
            answer += [rng.randrange(vocab) for _ in range(rng.randrange(1, 4))]
        traces.append({"prompt": prompt, "ops": ops})
    return traces


def _accept_cases(sp, rng: random.Random) -> list:
    out = []
    for _ in range(300):
        k = rng.randrange(0, 8)
        vocab = rng.choice([2, 4, 50])
        drafts = [rng.randrange(vocab) for _ in range(k)]
        arg = [d if rng.random() < 0.6 else rng.randrange(vocab) for d in drafts] + [rng.randrange(vocab)]
        out.append({"drafts": drafts, "argmax": arg, "result": sp.accept(drafts, arg)})
    return out


def _policy_trace(sp, cls_name: str, rng: random.Random) -> dict:
    rows = rng.choice([2, 4, 8, 16])
    policy = getattr(sp, cls_name)(rows)
    ops = []
    for _ in range(rng.randrange(20, 120)):
        r = rng.random()
        if r < 0.3:
            args = [rng.randrange(1, rows + 1), rng.choice([0.0, -1.0]) if rng.random() < 0.03
                    else round(rng.uniform(0.001, 0.2), 6), rng.random() < 0.5]
            policy.observe_step(*args)
            ops.append(["observe_step", args, None])
        elif r < 0.55:
            drafted = rng.randrange(0, 8)
            args = [rng.choice([2, 3, 102, 103, 104]), drafted, rng.randrange(0, drafted + 1)]
            policy.observe_drafts(*args)
            ops.append(["observe_drafts", args, None])
        elif r < 0.8:
            offers = [[[rng.randrange(100) for _ in range(rng.randrange(0, 8))], rng.choice([2, 3, 102, 104])]
                      for _ in range(rng.randrange(0, rows + 2))]
            ops.append(["choose", [offers], policy.choose([(o[0], o[1]) for o in offers])])
        elif r < 0.9:
            if cls_name == "WindowPolicy":
                which = rng.choice(["plain_price", "speculative_price", "price", "acceptance"])
            else:
                which = rng.choice(["price", "acceptance"])
            if which == "speculative_price":
                args = [rng.randrange(1, 20), rng.randrange(1, 8)]
            elif which == "acceptance":
                args = [rng.choice([2, 3, 102, 104])]
            else:
                args = [rng.randrange(1, 20)]
            ops.append([which, args, getattr(policy, which)(*args)])
        else:
            ops.append(["summary", [], policy.summary()])
    return {"rows": rows, "ops": ops}


def _collective_trace(sp, rng: random.Random) -> dict:
    keys = rng.choice([5, 50, 1000])
    index = sp.CollectiveIndex(keys=keys)
    ops = []
    for _ in range(rng.randrange(5, 40)):
        if rng.random() < 0.4:
            toks = [rng.randrange(12) for _ in range(rng.randrange(0, 20))]
            index.add(toks)
            ops.append(["add", [toks], None])
        else:
            ctx = [rng.randrange(12) for _ in range(rng.randrange(0, 8))]
            k = rng.randrange(0, 9)
            res = index.draft(ctx, k)
            ops.append(["draft", [ctx, k], [list(res[0]), res[1]]])
    ops.append(["len", [], len(index.table)])
    return {"keys": keys, "ops": ops}


def _draftstop_trace(dm, rng: random.Random) -> dict:
    stop = dm.DraftStop()
    ops = []
    for _ in range(rng.randrange(20, 100)):
        r = rng.random()
        if r < 0.2:
            confs = [round(rng.random(), 4) for _ in range(rng.randrange(0, 6))]
            args = [confs, rng.randrange(0, len(confs) + 1)]
            stop.learn(*args)
            ops.append(["learn", args, None])
        elif r < 0.35:
            args = [round(rng.uniform(0.001, 0.05), 6), rng.randrange(1, 5)]
            stop.observe_call(*args)
            ops.append(["observe_call", args, None])
        elif r < 0.5:
            running = rng.randrange(1, 4)
            args = [round(rng.uniform(0.01, 0.2), 6), running, rng.randrange(0, 5),
                    rng.choice([None, rng.randrange(1, 6)]), rng.choice([0.0, round(rng.uniform(0.001, 0.05), 6)])]
            stop.observe_step(*args)
            ops.append(["observe_step", args, None])
        elif r < 0.65:
            args = [rng.randrange(1, 4), rng.randrange(1, 3)]
            ops.append(["start", args, stop.start(*args)])
        elif r < 0.8:
            args = [round(rng.random(), 4), round(rng.uniform(0, 3), 4), round(rng.uniform(0, 0.1), 5),
                    rng.randrange(1, 4), rng.randrange(1, 3)]
            ops.append(["more", args, stop.more(*args)])
        elif r < 0.88:
            c = round(rng.random() * 1.1, 4)
            ops.append(["p", [c], stop.p(c)])
        elif r < 0.93:
            ops.append(["mean", [], stop.mean()])
        elif r < 0.97:
            rows = rng.randrange(1, 9)
            ops.append(["step_seconds", [rows], stop.step_seconds(rows)])
            ops.append(["call_seconds", [rows], stop.call_seconds(rows)])
        else:
            ops.append(["summary", [], stop.summary()])
    return {"ops": ops}


class _StandIn:
    """The reference's draft-engine stand-in protocol (tests/engine/test_draft_model.py:35-48), made
    deterministic from a seed: next token = (last + step) mod 997 with a confidence from a table."""

    def __init__(self, seqs: int, seed: int):
        import types

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


def _sig(tokens: list[int]) -> list[int]:
    """A compact signature of a token list: length, sum and the last 8 tokens."""
    return [len(tokens), sum(tokens), *tokens[-8:]]


class FixedClock:
    """time.perf_counter replaced by a clock that advances 4 ms per reading, so a trace of timed calls
    is reproducible. Used identically when the traces are replayed."""

    def __init__(self):
        self.now = 0.0

    def __call__(self) -> float:
        self.now += 0.004
        return self.now


def _drafter_trace(dm, rng: random.Random, seed: int) -> dict:
    """A drafter over a stand-in engine, timing replaced by a fixed clock so the trace is reproducible."""
    import time

    real, time.perf_counter = time.perf_counter, FixedClock()
    try:
        return _drafter_trace_timed(dm, rng, seed)
    finally:
        time.perf_counter = real


def _drafter_trace_timed(dm, rng: random.Random, seed: int) -> dict:
    engine = _StandIn(seqs=rng.choice([1, 2, 3]), seed=seed)
    drafter = dm.Drafter(engine, max_running=rng.choice([1, 2, 3]))
    ops = []
    texts: dict[int, list[int]] = {}
    for _ in range(rng.randrange(5, 25)):
        r = rng.random()
        if r < 0.6:
            wants = {}
            for key in rng.sample(range(5), rng.randrange(1, 3)):
                length = rng.randrange(260, 600) if rng.random() < 0.1 else rng.randrange(2, 40)
                base = texts.setdefault(key, [rng.randrange(997) for _ in range(length)])
                if rng.random() < 0.5:
                    base.extend(rng.randrange(997) for _ in range(rng.randrange(1, 4)))
                wants[key] = (list(base), rng.randrange(1, 6))
            running = rng.randrange(1, 4)
            res = drafter.draft(wants, running)
            ops.append(["draft", [{str(k): [v[0], v[1]] for k, v in wants.items()}, running],
                        {str(k): v for k, v in res.items()}])
        elif r < 0.85 and drafter._pending:
            key = rng.choice(sorted(drafter._pending))
            used = rng.randrange(0, 6)
            accepted = rng.randrange(0, used + 1)
            drafter.settle(key, used, accepted)
            ops.append(["settle", [key, used, accepted], None])
        elif r < 0.95:
            key = rng.randrange(5)
            drafter.release(key)
            ops.append(["release", [key], None])
        else:
            ops.append(["state", [], None])
        ops[-1].append({"held": {str(s): _sig(h) for s, h in drafter.held.items()},
                        "slot_of": {str(k): v for k, v in drafter.slot_of.items()},
                        "calls": len(engine.calls)})
    return {"seqs": engine.seqs, "max_running": drafter.max_running, "seed": seed, "ops": ops,
            "engine_calls": [[_sig(list(r)) for r in call] for call in engine.calls], "engine_removed": engine.removed,
            "stop_summary": {k: v for k, v in drafter.stop.summary().items() if "ms" not in k and "tok_s" not in k}}


def make_host() -> None:
    sp, dm = _load_reference_host()
    rng = random.Random(20261201)
    doc = {
        "constants": {"MAX_DRAFT": sp.MAX_DRAFT, "MIN_NGRAM": sp.MIN_NGRAM, "MAX_NGRAM": sp.MAX_NGRAM,
                      "POLICY_VERSION": sp.POLICY_VERSION, "MARGIN": sp.MARGIN,
                      "COLLECTIVE_BUCKET": sp.COLLECTIVE_BUCKET, "BINS": dm.BINS, "CHUNK": dm.CHUNK},
        "draft": _draft_cases(sp, rng),
        "ngram_index": _ngram_cases(sp, rng),
        "accept": _accept_cases(sp, rng),
        "window_policy": [_policy_trace(sp, "WindowPolicy", rng) for _ in range(60)],
        "step_policy": [_policy_trace(sp, "StepPolicy", rng) for _ in range(60)],
        "collective": [_collective_trace(sp, rng) for _ in range(40)],
        "draft_stop": [_draftstop_trace(dm, rng) for _ in range(40)],
        "drafter": [_drafter_trace(dm, rng, seed) for seed in range(24)],
        "suggest_draft": {name: dm.suggest_draft(name) for name in (
            "/models/Qwen3-4B-Q4_K_M.gguf", "Meta-Llama-3.1-8B-Instruct-Q4_K_M.gguf", "gemma-3-4b-it-Q4_K_M.gguf",
            "Qwen3-0.6B-Q8_0.gguf", "Mistral-7B-Instruct-v0.3-Q4_K_M.gguf", "C:\\m\\qwen3_14b.gguf",
            "llama-3.1-70b.gguf", "Llama-3.2-1B-Instruct-Q8_0.gguf")},
    }
    path = HERE / "host_traces.json"
    path.write_text(json.dumps(doc, separators=(",", ":")))
    print(path, path.stat().st_size)


if __name__ == "__main__":
    what = sys.argv[1:] or ["qmv", "host"]
    if "qmv" in what:
        make_qmv()
    if "host" in what:
        make_host()
