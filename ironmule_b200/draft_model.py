"""Speculation with a small draft model, stopped by a myopic optimal rule learned online.

The drop-in counterpart of IronMule's `ironmule/draft_model.py` (DraftStop :24-143, Drafter :159-288, DRAFTS and
suggest_draft :293-305): the same public names, the same engine protocol -- `_decode_conf(rows) -> [(token,
confidence)]`, `eog(token)`, `L.llama_memory_seq_rm(memory, seq, p0, p1)`, `memory`, `seqs` -- and the same
decisions, pinned by traces recorded from the reference (tests/golden/host_traces.json). The code is organised
around its own parts:

  _Calibration   a draft's chance of acceptance by the confidence bin of its top-1 probability (pseudo-counts)
  _Timing        seconds of draft-model calls by rows and of target steps by rows, with a line fitted through them
  _Payoff        measured tokens/s of steps with drafts per running-request count, and when to probe again
  DraftStop      the rule: draft at all (`start`), one more draft (`more`), built from the three above
  _SlotBook      which tokens each draft-model KV slot holds and which request owns which slot
  _EngineLink    the draft engine behind the protocol: timed decode calls and cache trims
  _Lane          one request's drafts, confidences and running acceptance chance within a draft step
  Drafter        a step: claim slots, catch each slot up with its request, then rounds of one draft row per
                 continuing request until the rule stops them; `settle` trims what the target rejected

`engine.DeviceDraftEngine` implements the protocol on the B200: `_decode_conf` runs the draft model on the device
and returns the argmax and the top-1 probability from `kernels.argmax_rows` (the device form of the reference's
host scan, ironmule/ggml_engine.py:669-683).
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Any, Sequence

BINS = 10
CHUNK = 256  # catch-up tokens one draft call carries at most
SMOOTH = 0.1  # weight of a new measurement in the running averages


def _blend(table: dict, key: int, value: float) -> None:
    """Running average of `value` under `key`: the first measurement, then moved SMOOTH of the way each time."""
    old = table.get(key)
    table[key] = value if old is None else old + SMOOTH * (value - old)


def _common(a: Sequence[int], b: Sequence[int]) -> int:
    """Length of the longest common prefix (64-token slices compared first, then token by token)."""
    if type(a) is not type(b):
        a, b = list(a), list(b)
    end = min(len(a), len(b))
    n = 0
    while n + 64 <= end and a[n:n + 64] == b[n:n + 64]:
        n += 64
    while n < end and a[n] == b[n]:
        n += 1
    return n


# ---- the stopping rule ---------------------------------------------------------------------------------------
class _Calibration:
    """A draft's chance of acceptance by its confidence bin. Pseudo-counts start every bin at its midpoint with
    weight 2, except the most confident bin (16 of 20), so the overall mean starts near 0.7."""

    def __init__(self) -> None:
        self.tried = [2.0] * BINS
        self.taken = [2.0 * (b + 0.5) / BINS for b in range(BINS)]
        self.tried[BINS - 1], self.taken[BINS - 1] = 20.0, 16.0

    @staticmethod
    def bin_of(confidence: float) -> int:
        return min(BINS - 1, max(0, int(confidence * BINS)))

    def chance(self, confidence: float) -> float:
        b = self.bin_of(confidence)
        return self.taken[b] / self.tried[b]

    def overall(self) -> float:
        return sum(self.taken) / sum(self.tried)

    def record(self, confidences: Sequence[float], accepted: int) -> None:
        """The target kept the first `accepted` drafts: those were tried and taken, the next one only tried."""
        for i, confidence in enumerate(confidences[:accepted + 1]):
            b = self.bin_of(confidence)
            self.tried[b] += 1
            self.taken[b] += i < accepted

    def table(self) -> list[float]:
        return [round(t / n, 3) for t, n in zip(self.taken, self.tried)]


class _Timing:
    """Seconds of draft-model calls by rows, and of target steps by rows with a least-squares line through them
    (a first-row cost and a per-row cost) for row counts not measured yet."""

    DEFAULT_STEP, DEFAULT_ROW, MIN_ROW = 0.085, 0.0025, 0.0005
    DEFAULT_CALL, CALL_ROW = 0.015, 0.001

    def __init__(self) -> None:
        self.call: dict[int, float] = {}
        self.by_rows: dict[int, float] = {}

    def line(self) -> tuple[float, float]:
        """(seconds of a step's first row, seconds per further row)."""
        pts = list(self.by_rows.items())
        if len(pts) >= 2:
            n = len(pts)
            r_bar = sum(r for r, _ in pts) / n
            t_bar = sum(t for _, t in pts) / n
            spread = sum((r - r_bar) ** 2 for r, _ in pts)
            slope = self.DEFAULT_ROW
            if spread > 0:
                slope = max(self.MIN_ROW, sum((r - r_bar) * (t - t_bar) for r, t in pts) / spread)
            return max(1e-4, t_bar - slope * (r_bar - 1)), slope
        first = pts[0][1] - self.DEFAULT_ROW * (pts[0][0] - 1) if pts else self.DEFAULT_STEP
        return max(1e-4, first), self.DEFAULT_ROW

    def step(self, rows: int) -> float:
        seen = self.by_rows.get(rows)
        if seen is not None:
            return seen
        first, per_row = self.line()
        return first + per_row * (rows - 1)

    def draft_call(self, rows: int) -> float:
        seen = self.call.get(rows)
        if seen is not None:
            return seen
        if not self.call:
            return self.DEFAULT_CALL + self.CALL_ROW * (rows - 1)
        nearest = min(self.call, key=lambda n: abs(n - rows))
        return max(1e-4, self.call[nearest] + self.CALL_ROW * (rows - nearest))


class _Payoff:
    """Tokens per second measured over steps that carried drafts, per running-request count. Once drafting has been
    measured (TRUST steps) to make fewer tokens/s than plain steps would, it is skipped, except on every PROBE-th
    ask, which measures again."""

    PROBE, TRUST = 25, 8

    def __init__(self) -> None:
        self.rate: dict[int, list[float]] = {}   # running -> [tokens/s, steps measured]
        self.asked: dict[int, int] = {}

    def losing(self, running: int, plain_rate: float) -> bool:
        self.asked[running] = self.asked.get(running, 0) + 1
        seen = self.rate.get(running)
        return (seen is not None and seen[1] >= self.TRUST and seen[0] < plain_rate
                and self.asked[running] % self.PROBE != 0)

    def record(self, running: int, tokens_per_second: float) -> None:
        seen = self.rate.setdefault(running, [tokens_per_second, 0])
        seen[0] += SMOOTH * (tokens_per_second - seen[0])
        seen[1] += 1


class DraftStop:
    """When to draft, and when to stop. A step with drafts pays off when its expected tokens per second beat a plain
    step's: start if (running + sharers x mean acceptance) / (step + draft call) beats running / step; add one more
    draft to a request while its marginal tokens per draft-second (chance all its drafts hold x mean acceptance /
    per-request draft cost) beat the step's expected tokens per second so far."""

    PROBE, TRUST = _Payoff.PROBE, _Payoff.TRUST

    def __init__(self) -> None:
        self.calibration = _Calibration()
        self.timing = _Timing()
        self.payoff = _Payoff()
        self.drafted = self.accepted = self.calls = self.steps = 0

    # the quantities the rule reads
    def p(self, confidence: float) -> float:
        return self.calibration.chance(confidence)

    def mean(self) -> float:
        return self.calibration.overall()

    @property
    def c_row(self) -> float:
        return self.timing.line()[1]

    def step_seconds(self, rows: int) -> float:
        return self.timing.step(rows)

    def call_seconds(self, rows: int) -> float:
        return self.timing.draft_call(rows)

    # the rule
    def start(self, running: int, sharers: int = 1) -> bool:
        """Draft in this step at all?"""
        plain = running / self.step_seconds(running)
        if self.payoff.losing(running, plain):
            return False
        cost = self.call_seconds(sharers) + self.c_row * sharers
        return (running + sharers * self.mean()) / (self.step_seconds(running) + cost) > plain

    def more(self, q: float, expected: float, spent: float, running: int, sharers: int) -> bool:
        """One more draft for a request whose drafts so far all hold with chance `q`?"""
        per_draft = self.call_seconds(sharers) / max(1, sharers) + self.c_row
        return q * self.mean() / per_draft > (running + expected) / (self.step_seconds(running) + spent)

    # what it learns from
    def learn(self, confidences: Sequence[float], accepted: int) -> None:
        self.calibration.record(confidences, accepted)
        self.drafted += len(confidences)
        self.accepted += accepted

    def observe_call(self, seconds: float, rows: int = 1) -> None:
        _blend(self.timing.call, rows, seconds)
        self.calls += 1

    def observe_step(self, seconds: float, running: int, draft_rows: int, tokens: int | None = None,
                     draft_seconds: float = 0.0) -> None:
        _blend(self.timing.by_rows, running + draft_rows, seconds)
        if draft_seconds > 0 and tokens is not None:
            self.payoff.record(running, tokens / (seconds + draft_seconds))
        self.steps += 1

    def summary(self) -> dict[str, Any]:
        first, per_row = self.timing.line()
        return {"drafted": self.drafted, "accepted": self.accepted, "draft_calls": self.calls,
                "acceptance_by_confidence": self.calibration.table(),
                "draft_call_ms_by_rows": {str(n): round(1000 * t, 1) for n, t in sorted(self.timing.call.items())},
                "step_ms": round(1000 * first, 1), "row_ms": round(1000 * per_row, 2),
                "tok_s_with_drafts_by_requests": {str(n): round(r[0], 1)
                                                  for n, r in sorted(self.payoff.rate.items())}}


# ---- the draft model's slots and calls ------------------------------------------------------------------------
Row = tuple[int, int, int, bool]  # (token, position, slot, wants logits)


class _EngineLink:
    """The draft engine behind the protocol: decode calls, timed (the seconds feed the stop rule), and trims of a
    slot's cache. `spent` is the draft-model seconds of the step being built and `catchup` the part of them that
    only read a request's new context (paid once per request, so left out of the check whether drafting pays)."""

    def __init__(self, engine: Any, stop: DraftStop):
        self.engine, self.stop = engine, stop
        self.spent = self.catchup = 0.0

    def decode(self, rows: list[Row], catchup: float = 0.0) -> list[tuple[int, float]]:
        """One call; `catchup` is the share of its rows that only read context. A call whose every row drafts
        times the draft call itself."""
        t0 = time.perf_counter()
        picks = self.engine._decode_conf(rows)
        seconds = time.perf_counter() - t0
        self.spent += seconds
        self.catchup += seconds * catchup
        if len(picks) == len(rows):
            self.stop.observe_call(seconds, len(rows))
        return picks

    def trim(self, slot: int, keep: int) -> bool:
        """Drop the slot's cells from `keep` on (False: the cache could not)."""
        return bool(self.engine.L.llama_memory_seq_rm(self.engine.memory, slot, keep, -1))

    def clear(self, slot: int) -> None:
        self.engine.L.llama_memory_seq_rm(self.engine.memory, slot, -1, -1)


class _SlotBook:
    """Which tokens each draft-model KV slot holds (`held`) and which request owns which slot (`slot_of`). A request
    takes the free slot sharing the longest prefix with its context; a finished request's slot keeps its cells."""

    def __init__(self, slots: int):
        self.held: dict[int, list[int]] = {s: [] for s in range(slots)}
        self.slot_of: dict[int, int] = {}

    def claim(self, key: int, context: Sequence[int]) -> bool:
        if key in self.slot_of:
            return True
        owned = set(self.slot_of.values())
        free = [s for s in self.held if s not in owned]
        if not free:
            return False
        self.slot_of[key] = max(free, key=lambda s: _common(self.held[s], context))
        return True

    def sync(self, slot: int, context: Sequence[int], link: _EngineLink) -> list[Row]:
        """Bring the slot up to `context`. Cells past the shared prefix go (the context's last token is always
        recomputed, for its logits); a cache that cannot cut there is cleared. Long catch-ups go in CHUNK-token calls
        of their own; the rows of the rest are returned, the last one wanting logits."""
        held = self.held[slot]
        keep = min(_common(held, context), len(context) - 1)
        if len(held) > keep:
            if keep == 0 or not link.trim(slot, keep):
                link.clear(slot)
                keep = 0
            del held[keep:]
        rest = context[keep:]
        while len(rest) > CHUNK:
            chunk, rest = rest[:CHUNK], rest[CHUNK:]
            link.decode([(tok, len(held) + i, slot, False) for i, tok in enumerate(chunk)], catchup=1.0)
            held.extend(chunk)
        rows = [(tok, len(held) + i, slot, i == len(rest) - 1) for i, tok in enumerate(rest)]
        held.extend(rest)
        return rows

    def extend(self, slot: int, token: int) -> Row:
        """The row that feeds one more draft to the slot (its cell is held from now on)."""
        row = (token, len(self.held[slot]), slot, True)
        self.held[slot].append(token)
        return row


@dataclass
class _Lane:
    """One request in a draft step."""
    key: int
    slot: int
    room: int                       # drafts it has room for
    context_len: int
    drafts: list[int] = field(default_factory=list)
    confidences: list[float] = field(default_factory=list)
    chance: float = 1.0             # that every draft so far is accepted
    pick: tuple[int, float] = (0, 0.0)  # the draft model's next token and its confidence


class Drafter:
    """Drafts for the running requests from a draft model behind the reference's engine protocol (a
    `DeviceDraftEngine` on the B200, or any stand-in with `_decode_conf`, `eog`, `L`, `memory` and `seqs`)."""

    def __init__(self, engine: Any, max_running: int = 2):
        self.e = engine
        self.max_running = max_running  # beyond this many running requests the draft model rests
        self.stop = DraftStop()
        self.book = _SlotBook(engine.seqs)
        self.link = _EngineLink(engine, self.stop)
        self._pending: dict[int, tuple[int, list[float]]] = {}  # key -> (context length, confidences of its drafts)

    # the state the reference exposes under these names
    @property
    def held(self) -> dict[int, list[int]]:
        return self.book.held

    @property
    def slot_of(self) -> dict[int, int]:
        return self.book.slot_of

    @property
    def step_seconds(self) -> float:
        return self.link.spent

    @property
    def catchup_seconds(self) -> float:
        return self.link.catchup

    def release(self, key: int) -> None:
        """The request ended; its slot keeps its cells for a later request with the same prefix."""
        self.book.slot_of.pop(key, None)
        self._pending.pop(key, None)

    def draft(self, wants: dict[int, tuple[Sequence[int], int]], running: int) -> dict[int, list[int]]:
        """Drafts for the requests in `wants` (key -> (tokens so far, room for drafts)), as many as the rule allows;
        {} where it gives none. `running` is the number of requests in the step."""
        link, book = self.link, self.book
        link.spent = link.catchup = 0.0
        if running > self.max_running:
            return {}
        lanes = [_Lane(key, book.slot_of[key], room, len(ctx)) for key, (ctx, room) in wants.items()
                 if book.claim(key, ctx)]
        if not lanes or not self.stop.start(running, len(lanes)):
            return {}
        tails: list[Row] = []
        for lane in lanes:
            tails += book.sync(lane.slot, wants[lane.key][0], link)
        for lane, pick in zip(lanes, link.decode(tails, catchup=(len(tails) - len(lanes)) / max(1, len(tails)))):
            lane.pick = pick
        self._rounds(lanes, running)
        for lane in lanes:
            self._pending[lane.key] = (lane.context_len, lane.confidences)
        return {lane.key: lane.drafts for lane in lanes}

    def _rounds(self, lanes: list[_Lane], running: int) -> None:
        """Take each lane's pick as a draft; lanes with room left and no end token ask the rule for one more; those
        it allows get one draft row each in the next call."""
        expected, spent, active = 0.0, self.link.spent, lanes
        while active:
            room_left = []
            for lane in active:
                token, confidence = lane.pick
                lane.drafts.append(token)
                lane.confidences.append(confidence)
                lane.chance *= self.stop.p(confidence)
                expected += lane.chance
                if len(lane.drafts) < lane.room and not self.e.eog(token):
                    room_left.append(lane)
            active = [lane for lane in room_left
                      if self.stop.more(lane.chance, expected, spent, running, len(room_left))]
            if not active:
                return
            picks = self.link.decode([self.book.extend(lane.slot, lane.drafts[-1]) for lane in active])
            spent = self.link.spent + self.stop.c_row * sum(len(lane.drafts) for lane in lanes)
            for lane, pick in zip(active, picks):
                lane.pick = pick

    def settle(self, key: int, used: int, accepted: int) -> None:
        """The target verified the request's first `used` drafts and kept `accepted` of them: the rule learns from
        it, and the slot's cells past what still matches the text go."""
        pending = self._pending.pop(key, None)
        slot = self.book.slot_of.get(key)
        if pending is None or slot is None:
            return
        context_len, confidences = pending
        self.stop.learn(confidences[:used], accepted)
        held = self.book.held[slot]
        keep = context_len + min(accepted, max(0, len(held) - context_len))
        if len(held) > keep:
            self.link.trim(slot, keep)
            del held[keep:]

    def end_step(self, seconds: float, running: int, draft_rows: int, tokens: int) -> None:
        """The step the drafts were for took `seconds` and made `tokens` tokens."""
        drafting = max(1e-6, self.link.spent - self.link.catchup) if draft_rows else 0.0
        self.stop.observe_step(seconds, running, draft_rows, tokens, drafting)
        self.link.spent = self.link.catchup = 0.0

    def summary(self) -> dict[str, Any]:
        return {"slots": len(self.book.held), "max_running": self.max_running, **self.stop.summary()}

    def close(self) -> None:
        close = getattr(self.e, "close", None)
        if close is not None:
            close()


# Draft models known to pair with a target family: (family, repository, file).
DRAFTS = (("qwen3", "Qwen/Qwen3-0.6B-GGUF", "Qwen3-0.6B-Q8_0.gguf"),
          ("llama-3.1", "bartowski/Llama-3.2-1B-Instruct-GGUF", "Llama-3.2-1B-Instruct-Q8_0.gguf"))


def suggest_draft(gguf: str) -> dict[str, str] | None:
    """A draft model of the same family as `gguf` (by file name) and the command that would fetch it."""
    name = gguf.replace("\\", "/").rsplit("/", 1)[-1].lower().replace("_", "-")
    for family, repo, file in DRAFTS:
        if family in name and file.lower().replace("_", "-") not in name:
            return {"repo": repo, "file": file,
                    "download": f"curl -L -o {file} https://huggingface.co/{repo}/resolve/main/{file}",
                    "use": f"--draft-gguf {file}"}
    return None


__all__ = ["DRAFTS", "DraftStop", "Drafter", "suggest_draft"]
