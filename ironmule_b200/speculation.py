"""Context speculation: n-gram drafting, greedy acceptance and the learned draft-window policies.

The drop-in counterpart of IronMule's `ironmule/speculation.py` (same names, arguments, results and
errors). Drafting copies the tokens that followed the most recent earlier occurrence of the context's
longest repeated suffix; acceptance keeps the drafts up to the first one the target disagrees with, then the
target's own token; the policies decide how many drafts each request of a step gets, from this machine's
measured step times and this traffic's measured acceptance.

On the B200 engine these run on the host between device rounds; the per-token work of a round (argmax,
acceptance, KV rollback) runs on the device (`ironmule_b200.kernels.verify_greedy`, `engine`).

Reference: ironmule/speculation.py:28-36 (constants), :39-53 (draft), :56-100 (NgramIndex),
:103-108 (accept), :111-230 (WindowPolicy), :233-322 (StepPolicy), :328-374 (CollectiveIndex).
"""
from __future__ import annotations

import threading
from collections import OrderedDict
from typing import Any, Sequence

POLICY_VERSION = 2
MAX_DRAFT = 7
MAX_NGRAM = 3
MIN_NGRAM = 2
LINE_MEMORY = 50          # a new speculative step weighs as much as the last 50 together
PRIOR_ACCEPT, PRIOR_WEIGHT = 0.3, 4.0
COST_WEIGHT = 0.2         # exponential weight of a new plain step
ROW_SLOPE = 0.06          # prior relative cost of one more row
MARGIN = 1.02
COLLECTIVE_BUCKET = 100
COLLECTIVE_NGRAM = 4


def _tail_matches(context: Sequence[int], start: int, n: int) -> bool:
    """context[start:start+n] equals the last n tokens of context."""
    end = len(context) - n
    return all(context[start + i] == context[end + i] for i in range(n))


def draft(context: Sequence[int], k: int, max_ngram: int = MAX_NGRAM,
          min_ngram: int = MIN_NGRAM) -> tuple[list[int], int]:
    """Up to `k` tokens that followed the most recent earlier occurrence of the longest suffix (from
    `max_ngram` down to `min_ngram` tokens) that repeats in `context`, and that suffix's length; ([], 0)
    when no suffix repeats."""
    if k < 1:
        return [], 0
    size = len(context)
    n = min(max_ngram, size - 1)
    while n >= min_ngram:
        for start in range(size - n - 1, -1, -1):
            if _tail_matches(context, start, n):
                following = list(context[start + n:start + n + k])
                if following:
                    return following, n
        n -= 1
    return [], 0


class NgramIndex:
    """`draft` by table lookup: for every n, the last start of each n-gram in the request's tokens, kept
    current as the answer grows, so a lookup costs O(1) per n whatever the context length and each token is
    indexed once. `draft(k)` returns exactly `draft(tokens, k)`."""

    __slots__ = ("tokens", "max_ngram", "min_ngram", "_last", "_done", "_base")

    def __init__(self, prompt: Sequence[int], max_ngram: int = MAX_NGRAM, min_ngram: int = MIN_NGRAM):
        self.tokens = list(prompt)
        self.max_ngram, self.min_ngram = max_ngram, min_ngram
        self._last: dict[int, dict[tuple[int, ...], int]] = {n: {} for n in range(min_ngram, max_ngram + 1)}
        self._done = 0             # n-grams ending before this position are indexed
        self._base = len(self.tokens)

    def follow(self, answer: Sequence[int]) -> None:
        """Take the tokens of `answer` (which only grows) not seen yet."""
        have = len(self.tokens) - self._base
        if len(answer) > have:
            self.tokens.extend(answer[have:])

    def append(self, token: int) -> None:
        self.tokens.append(token)

    def _index(self) -> None:
        # Every n-gram ending at positions [_done, len-1): the one ending at the last token is the suffix
        # itself, not an earlier occurrence.
        tokens, stop = self.tokens, len(self.tokens) - 1
        for end in range(self._done, stop):
            for n, table in self._last.items():
                first = end - n + 1
                if first >= 0:
                    table[tuple(tokens[first:end + 1])] = first
        self._done = max(self._done, stop)

    def draft(self, k: int) -> tuple[list[int], int]:
        if k < 1:
            return [], 0
        self._index()
        tokens, size = self.tokens, len(self.tokens)
        for n in range(min(self.max_ngram, size - 1), self.min_ngram - 1, -1):
            first = self._last[n].get(tuple(tokens[size - n:]))
            if first is not None:
                following = tokens[first + n:first + n + k]
                if following:
                    return following, n
        return [], 0


def accept(drafts: Sequence[int], argmax: Sequence[int]) -> list[int]:
    """The leading drafts equal to the target's argmax at their position, then the target's own token."""
    agreed = 0
    for d, a in zip(drafts, argmax):
        if d != a:
            break
        agreed += 1
    return list(drafts[:agreed]) + [int(argmax[agreed])]


def _prior_scaled(seconds_at: float, rows_at: int, rows: int) -> float:
    """A measured price at `rows_at` rows carried to `rows` rows by the prior slope."""
    return seconds_at * (1.0 + ROW_SLOPE * (rows - 1)) / (1.0 + ROW_SLOPE * (rows_at - 1))


def _greedy_windows(offers, rates, rate0, tokens0, rows0, budget, price_of) -> tuple[list[int], float]:
    """Hand out drafts one at a time to the request whose next draft adds the most expected tokens, while
    the step's expected tokens per second (`price_of(rows)` seconds for `rows` rows) keeps rising."""
    ks = [0] * len(offers)
    reach = [1.0] * len(offers)
    tokens, rows, rate = tokens0, rows0, rate0
    while budget > 0:
        best, gain = None, 0.0
        for i, (drafts, _) in enumerate(offers):
            if ks[i] < len(drafts):
                add = reach[i] * rates[i]
                if add > gain:
                    best, gain = i, add
        if best is None:
            break
        new_rate = (tokens + gain) / price_of(rows + 1)
        if new_rate <= rate:
            break
        ks[best] += 1
        reach[best] *= rates[best]
        tokens, rows, rate, budget = tokens + gain, rows + 1, new_rate, budget - 1
    return ks, rate


class _AcceptanceBook:
    """Per-bucket counts of drafts tried and taken, with the prior (0.3 worth 4 drafts)."""

    def _init_book(self) -> None:
        self.tried: dict[int, float] = {}
        self.taken: dict[int, float] = {}
        self.steps = self.plain_steps = self.drafted = self.accepted = 0
        self._lock = threading.Lock()

    def acceptance(self, bucket: int) -> float:
        with self._lock:
            tried, taken = self.tried.get(bucket, 0.0), self.taken.get(bucket, 0.0)
        return (taken + PRIOR_ACCEPT * PRIOR_WEIGHT) / (tried + PRIOR_WEIGHT)

    def observe_drafts(self, bucket: int, drafted: int, accepted: int) -> None:
        """`accepted` of `drafted` drafts were kept; the first refused one counts as tried, later ones not."""
        if drafted < 1:
            return
        with self._lock:
            reached = accepted + (1 if accepted < drafted else 0)
            self.tried[bucket] = self.tried.get(bucket, 0.0) + reached
            self.taken[bucket] = self.taken.get(bucket, 0.0) + accepted
            self.drafted += drafted
            self.accepted += accepted

    def _acceptance_summary(self) -> dict[str, float]:
        buckets = sorted(set(self.tried) | set(self.taken))
        return {str(b): round(self.acceptance(b), 4) for b in buckets}


class WindowPolicy(_AcceptanceBook):
    """Drafts per request for a stacked plan whose plain and speculative steps cost differently (policy
    version 2): plain steps priced per row count by an exponential average, speculative steps by a decayed
    least-squares line through every speculative step."""

    def __init__(self, rows: int):
        if rows < 1:
            raise ValueError("a step needs at least one row")
        self.rows = rows
        self.plain: dict[int, float] = {}
        self._line = [0.0] * 5  # decayed sums of w, w*r, w*r*r, w*t, w*r*t
        self._line_rows: set[int] = set()
        self._init_book()

    def plain_price(self, rows: int) -> float:
        with self._lock:
            if rows in self.plain:
                return self.plain[rows]
            nearest = None
            for r, t in self.plain.items():  # first-inserted wins a tie in distance
                if nearest is None or abs(r - rows) < abs(nearest[0] - rows):
                    nearest = (r, t)
        if nearest is None:
            return 1.0 + ROW_SLOPE * (rows - 1)
        return _prior_scaled(nearest[1], nearest[0], rows)

    def speculative_price(self, rows: int, requests: int) -> float:
        with self._lock:
            w, wr, wrr, wt, wrt = self._line
            fitted = len(self._line_rows) >= 2
        if not fitted:
            return self.plain_price(requests) * (1.0 + ROW_SLOPE * (rows - requests))
        spread = w * wrr - wr * wr
        slope = max(0.0, (w * wrt - wr * wt) / spread) if spread > 0 else 0.0
        return max(1e-6, (wt - slope * wr) / w + slope * rows)

    def price(self, rows: int) -> float:
        return self.plain_price(rows)

    def choose(self, offers: Sequence[tuple[Sequence[int], int]]) -> list[int]:
        """Drafts per request; never more than offered or than the plan's free rows. All zeros = plain."""
        n = len(offers)
        budget = self.rows - n
        if n == 0 or budget <= 0 or not any(tokens for tokens, _ in offers):
            return [0] * n
        rates = [self.acceptance(bucket) for _, bucket in offers]
        ks, rate = _greedy_windows(offers, rates, n / self.speculative_price(n, n), float(n), n, budget,
                                   lambda rows: self.speculative_price(rows, n))
        if not any(ks) or rate < MARGIN * n / self.plain_price(n):
            return [0] * n
        return ks

    def observe_step(self, rows: int, seconds: float, speculative: bool) -> None:
        if not (seconds > 0) or rows < 1:
            return
        with self._lock:
            if speculative:
                keep = 1.0 - 1.0 / LINE_MEMORY
                point = (1.0, rows, rows * rows, seconds, rows * seconds)
                self._line = [old * keep + add for old, add in zip(self._line, point)]
                self._line_rows.add(rows)
                self.steps += 1
            else:
                old = self.plain.get(rows)
                self.plain[rows] = seconds if old is None else (1 - COST_WEIGHT) * old + COST_WEIGHT * seconds
                self.plain_steps += 1

    def summary(self) -> dict[str, Any]:
        with self._lock:
            plain = {str(r): round(t * 1000, 3) for r, t in sorted(self.plain.items())}
            counts = (self.steps, self.plain_steps, self.drafted, self.accepted)
            fitted = len(self._line_rows) >= 2
            acceptance_keys = sorted(set(self.tried) | set(self.taken))
        line = ({str(r): round(self.speculative_price(r, 1) * 1000, 3) for r in range(1, self.rows + 1)}
                if fitted else {})
        return {"policy": "context", "policy_version": POLICY_VERSION, "speculative_steps": counts[0],
                "plain_steps": counts[1], "drafted": counts[2], "accepted": counts[3],
                "acceptance": {str(b): round(self.acceptance(b), 4) for b in acceptance_keys},
                "plain_step_ms_by_rows": plain, "speculative_step_ms_by_rows": line}


class StepPolicy(_AcceptanceBook):
    """Drafts per request for an engine whose every step is one call priced by its rows (policy version 3):
    a row count's price is the median of its last WINDOW steps once it has PROBES of them, else the nearest
    measured count scaled by the prior slope, so a size is tried before a guessed price can veto it."""

    WINDOW, PROBES, VERSION = 16, 3, 3

    def __init__(self, rows: int):
        if rows < 1:
            raise ValueError("a step needs at least one row")
        self.rows = rows
        self.times: dict[int, list[float]] = {}
        self._init_book()

    def price(self, rows: int) -> float:
        with self._lock:
            measured = {r: sorted(t)[len(t) // 2] for r, t in self.times.items() if len(t) >= self.PROBES}
        if rows in measured:
            return measured[rows]
        if not measured:
            return 1.0 + ROW_SLOPE * (rows - 1)
        near = min(measured, key=lambda r: (abs(r - rows), r))
        return _prior_scaled(measured[near], near, rows)

    def choose(self, offers: Sequence[tuple[Sequence[int], int]]) -> list[int]:
        n = len(offers)
        budget = self.rows - n
        if n == 0 or budget <= 0 or not any(tokens for tokens, _ in offers):
            return [0] * n
        rates = [self.acceptance(bucket) for _, bucket in offers]
        plain = n / self.price(n)
        ks, rate = _greedy_windows(offers, rates, plain, float(n), n, budget, self.price)
        return ks if any(ks) and rate >= MARGIN * plain else [0] * n

    def observe_step(self, rows: int, seconds: float, speculative: bool) -> None:
        if not (seconds > 0) or rows < 1:
            return
        with self._lock:
            window = self.times.setdefault(rows, [])
            window.append(seconds)
            del window[:-self.WINDOW]
            if speculative:
                self.steps += 1
            else:
                self.plain_steps += 1

    def summary(self) -> dict[str, Any]:
        with self._lock:
            counts = (self.steps, self.plain_steps, self.drafted, self.accepted)
            sizes = sorted(self.times)
            acceptance_keys = sorted(set(self.tried) | set(self.taken))
        return {"policy": "context", "policy_version": self.VERSION, "speculative_steps": counts[0],
                "plain_steps": counts[1], "drafted": counts[2], "accepted": counts[3],
                "acceptance": {str(b): round(self.acceptance(b), 4) for b in acceptance_keys},
                "step_ms_by_rows": {str(r): round(self.price(r) * 1000, 3) for r in sizes}}


class CollectiveIndex:
    """Drafts from other requests' answers: every `ngram`..2-gram of recent answers mapped to up to
    MAX_DRAFT tokens that followed it (the most recent answer wins), bounded to `keys` n-grams with the
    least recently written dropped first. Drafts from it are learned in bucket COLLECTIVE_BUCKET + n."""

    def __init__(self, keys: int = 200_000, ngram: int = COLLECTIVE_NGRAM):
        self.keys, self.ngram = keys, ngram
        self.table: OrderedDict[tuple[int, ...], tuple[int, ...]] = OrderedDict()
        self._lock = threading.Lock()
        self.added = 0

    def add(self, tokens: Sequence[int]) -> None:
        tokens = list(tokens)
        with self._lock:
            for n in range(self.ngram, 1, -1):
                for i in range(len(tokens) - n):
                    key = tuple(tokens[i:i + n])
                    self.table[key] = tuple(tokens[i + n:i + n + MAX_DRAFT])
                    self.table.move_to_end(key)
            while len(self.table) > self.keys:
                self.table.popitem(last=False)
            self.added += 1

    def draft(self, context: Sequence[int], k: int) -> tuple[list[int], int]:
        if k < 1:
            return [], 0
        with self._lock:
            for n in range(min(self.ngram, len(context)), 1, -1):
                found = self.table.get(tuple(context[len(context) - n:]))
                if found:
                    return list(found[:k]), COLLECTIVE_BUCKET + n
        return [], 0


__all__ = ["COLLECTIVE_BUCKET", "CollectiveIndex", "MARGIN", "MAX_DRAFT", "MIN_NGRAM", "NgramIndex",
           "POLICY_VERSION", "StepPolicy", "WindowPolicy", "accept", "draft"]
