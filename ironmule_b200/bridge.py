"""The product bridge's generation calls over the device engine: `generate` / `generate_many` of
ironmule_product/ggml_bridge.py:231-291, served by a continuous-batching loop with the reference engine's request
semantics (`GgmlEngine.run`, ironmule/ggml_engine.py:1000-1160).

`serve(decoder, jobs, admit, eog)` keeps the decoder's sequence slots busy: waiting requests start in idle slots
shortest prompt first (at least two prompt tokens: the device round re-feeds the last two), `admit(free slots)`
is asked for more whenever slots are free, and after every round each running request takes its new tokens one by
one, as the reference's `take` does (ggml_engine.py:1037-1056):
- a request whose `cancelled()` answers True ends as "cancelled";
- otherwise the token is appended and emitted, and the request ends as "eos" on an end-of-generation token or as
  "length" at its limit.
A request that ends frees its slot at once (`SpecDecoder.stop_slot`: with a page pool its K/V stay cached for
later requests with the same prefix). The decoder's round runs as one CUDA graph, captured after the first round.
Requests are checked when they arrive: invalid ones among those `serve` is called with raise before any slot starts;
an invalid one that `admit` hands over ends at once as "invalid" (its message in `error`) while the others run on. If
anything raises while requests run, their slots are stopped before the exception leaves `serve`.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Any, Callable, Sequence

import torch


@dataclass
class Job:
    """One request (the reference's `Job`, ironmule/ggml_engine.py:193-216): prompt ids, token limit, a callback
    per token, an optional cancel predicate; filled in by `serve`."""

    ids: list[int]
    limit: int
    emit: Callable[[int], None] | None = None
    cancelled: Callable[[], bool] | None = None
    tokens: list[int] = field(default_factory=list)
    reason: str | None = None
    reused: int = 0  # prompt tokens whose K/V were linked from the page pool instead of computed
    first_ns: int = 0
    finished_ns: int = 0
    error: str | None = None


def _invalid(job: Job, limit: int) -> str | None:
    """Why the decoder cannot serve the request, or None."""
    if len(job.ids) < 2 or job.limit < 1:
        return "a request needs at least two prompt tokens and a positive limit"
    if len(job.ids) + job.limit > limit:
        return f"{len(job.ids) + job.limit} tokens do not fit a {limit}-token sequence"
    return None


@dataclass
class BridgeResult:
    """The fields of the reference's `EngineBridgeResult` (ironmule_product/engine_bridge.py:23-31)."""

    tokens: list[int] = field(repr=False)
    text: str = field(repr=False)
    finish_reason: str
    token_count: int
    metrics: dict[str, Any] = field(repr=False)
    metadata: dict[str, Any]


def serve(dec, jobs: list[Job], admit: Callable[[int], list[Job]] | None = None,
          eog: Callable[[int], bool] = lambda token: False) -> list[Job]:
    """Serve `jobs`, and every job `admit(free slots)` hands over while they run, on `dec` (a `SpecDecoder` or
    anything with its `batch`, `start_slots`, `stop_slot`, `step`, `capture`, `graph`, `device` and
    `request_limit`); returns them all in arrival order."""
    limit = dec.request_limit()
    for job in jobs:
        why = _invalid(job, limit)
        if why is not None:
            raise ValueError(why)
    served, pending = list(jobs), list(jobs)
    active: dict[int, Job] = {}
    rounds = 0

    def arrive(more: list[Job]) -> None:
        served.extend(more)
        for job in more:
            why = _invalid(job, limit)
            if why is None:
                pending.append(job)
            else:
                job.reason, job.error, job.finished_ns = "invalid", why, time.monotonic_ns()

    def finish(slot: int, job: Job, reason: str) -> None:
        job.reason, job.finished_ns = reason, time.monotonic_ns()
        active.pop(slot)
        dec.stop_slot(slot)

    def take(slot: int, job: Job, token: int) -> bool:
        if job.cancelled is not None and job.cancelled():
            finish(slot, job, "cancelled")
            return True
        job.tokens.append(token)
        if job.first_ns == 0:
            job.first_ns = time.monotonic_ns()
        if job.emit is not None:
            job.emit(token)
        if eog(token):
            finish(slot, job, "eos")
            return True
        if len(job.tokens) >= job.limit:
            finish(slot, job, "length")
            return True
        return False

    try:
        return _loop(dec, admit, active, pending, arrive, take, served, rounds)
    except BaseException:
        for b in list(active):
            dec.stop_slot(b)
        raise


def _loop(dec, admit, active, pending, arrive, take, served, rounds) -> list[Job]:
    while True:
        free = [b for b in range(dec.batch) if b not in active]
        if admit is not None and free:
            arrive(admit(len(free)))
        fresh = []
        for job in sorted(pending, key=lambda j: len(j.ids)):
            if job.cancelled is not None and job.cancelled():
                job.reason, job.finished_ns = "cancelled", time.monotonic_ns()
                pending.remove(job)
                continue
            if not free:
                break
            pending.remove(job)
            fresh.append((free.pop(0), job))
        if fresh:
            dec.start_slots([(b, torch.tensor(job.ids, dtype=torch.int32, device=dec.device), job.limit)
                             for b, job in fresh])
            for b, job in fresh:
                job.reused = dec.reused[b]
                active[b] = job
        if not active:
            if pending:
                continue
            if admit is not None:
                more = admit(dec.batch)
                if more:
                    arrive(more)
                    continue
            return served
        if dec.graph is None and rounds == 1:
            dec.capture()  # after one eager round has loaded every kernel
        news = dec.step()
        rounds += 1
        for b, job in list(active.items()):
            for token in news.get(b, []):
                if take(b, job, token):
                    break


class DeviceBridge:
    """`generate` / `generate_many` and the bridge's small queries (ironmule_product/ggml_bridge.py:200-291) over a
    `SpecDecoder` (or `TreeDecoder`) whose slots serve the requests. `tokenizer` needs `decode(ids)`; `eos_ids`
    are the end-of-generation tokens. The reference's `boundaries` (multi-shot prompts) are refused, as its ggml
    bridge refuses them."""

    def __init__(self, decoder, tokenizer: Any = None, eos_ids: Sequence[int] = ()):
        self._dec = decoder
        self._tokenizer = tokenizer
        self._eos = tuple(int(t) for t in eos_ids)
        self._served = 0
        self._tokens = 0

    def eos_ids(self) -> tuple[int, ...]:
        return self._eos

    def request_limit(self) -> int:
        return self._dec.request_limit()

    def free_slots(self) -> int:
        return sum(1 for r in self._dec.running if not r)

    def metadata(self) -> dict[str, Any]:
        d = self._dec
        return {"configuration": "b200", "plan": "strict_one_shot",
                "b200": {"target": d.target.cfg.name, "draft": d.draft.cfg.name, "k": d.k, "slots": d.batch,
                         "prefix_cache": d.pool is not None,
                         "answers": "greedy decoding's tokens (speculation changes no answer)"}}

    def counters(self) -> dict[str, Any]:
        out: dict[str, Any] = {"requests": self._served, "tokens": self._tokens}
        if self._dec.pool is not None:
            out["prefix"] = self._dec.pool.summary()
        return out

    def generate(self, prompt_ids: Sequence[int], max_tokens: int, on_token=None,
                 boundaries: Sequence[int] | None = None) -> BridgeResult:
        return self.generate_many([prompt_ids], max_tokens, on_tokens=[on_token],
                                  boundaries=None if boundaries is None else [boundaries])[0]

    def generate_many(self, prompt_ids: Sequence[Sequence[int]], max_tokens: int | Sequence[int], on_tokens=None,
                      boundaries=None, admit: Callable[[int], list[Any]] | None = None,
                      cancelled=None) -> list[BridgeResult]:
        if boundaries is not None and any(cuts is not None for cuts in boundaries):
            raise ValueError("the device engine serves one-shot prompts")
        limits = [max_tokens] * len(prompt_ids) if type(max_tokens) is int else list(max_tokens)
        emitters = list(on_tokens) if on_tokens is not None else [None] * len(prompt_ids)
        stops = list(cancelled) if cancelled is not None else [None] * len(prompt_ids)
        jobs = [Job(list(ids), int(limit), emit, stop)
                for ids, limit, emit, stop in zip(prompt_ids, limits, emitters, stops)]

        def take(free: int) -> list[Job]:  # admit's rows: (ids, limit, emit[, boundaries[, cancelled]])
            fresh = []
            for row in admit(free):
                ids, limit, emit = row[:3]
                if len(row) > 3 and row[3] is not None:
                    raise ValueError("the device engine serves one-shot prompts")
                fresh.append(Job(list(ids), int(limit), emit, row[4] if len(row) > 4 else None))
            return fresh

        eos = set(self._eos)
        served = serve(self._dec, jobs, admit=take if admit is not None else None, eog=lambda t: t in eos)
        reasons = {"eos": "stop", "length": "length", "cancelled": "cancelled", "invalid": "error"}
        results = []
        for job in served:
            kept = [t for t in job.tokens if t not in eos]
            text = self._tokenizer.decode(kept) if self._tokenizer is not None else ""
            self._served += 1
            self._tokens += len(job.tokens)
            results.append(BridgeResult(tokens=list(job.tokens), text=text,
                                        finish_reason=reasons[job.reason or "cancelled"],
                                        token_count=len(job.tokens),
                                        metrics={"reused_prompt_tokens": job.reused,
                                                 "first_token_ns": job.first_ns, "finished_ns": job.finished_ns},
                                        metadata={**self.metadata(), **self.counters(),
                                                  **({"error": job.error} if job.error else {})}))
        return results

    def close(self) -> None:
        self._dec.finish(keep=False)
        self._dec.graph = None
