"""Speculation with a small draft model, stopped by a myopic optimal rule learned online.

The drop-in counterpart of IronMule's `ironmule/draft_model.py`: `DraftStop` (calibration of the draft
model's top-1 confidence into an acceptance chance, the machine's step and draft-call costs, and the
start / one-more-draft rule), `Drafter` (the draft model's KV slots kept in step with each request, the
catch-up in CHUNK-token calls, one draft row per request per call, KV trimmed on rejection) and
`suggest_draft`. The engine protocol is the reference's: `_decode_conf(rows) -> [(token, confidence)]`,
`eog(token)`, `L.llama_memory_seq_rm(memory, seq, p0, p1)`, `memory`, `seqs`.

`DeviceDraftEngine` (ironmule_b200.engine) implements that protocol on the B200: its `_decode_conf` runs
the draft model on the device and returns argmax and top-1 probability from `kernels.argmax_rows`, the
device form of the reference's host scan (ironmule/ggml_engine.py:669-683).

Reference: ironmule/draft_model.py:24-143 (DraftStop), :146-156 (_common), :159-288 (Drafter),
:293-305 (DRAFTS, suggest_draft).
"""
from __future__ import annotations

import time
from typing import Any, Sequence

BINS = 10
CHUNK = 256  # catch-up tokens one draft call carries at most


def _bin(confidence: float) -> int:
    return min(BINS - 1, max(0, int(confidence * BINS)))


class DraftStop:
    """The stopping rule's state: acceptance by confidence bin, draft-call seconds by rows, step seconds by
    rows (fitted to a line), and per running-request count the measured tokens/s of steps with drafts.
    Where drafting measured slower than plain steps it stops, and is probed again once every PROBE steps."""

    PROBE, TRUST = 25, 8

    def __init__(self) -> None:
        self.tried = [2.0] * BINS
        self.taken = [2.0 * (i + 0.5) / BINS for i in range(BINS)]
        self.tried[-1], self.taken[-1] = 20.0, 16.0  # confident drafts dominate: the mean starts near 0.7
        self.call: dict[int, float] = {}
        self.by_rows: dict[int, float] = {}
        self.rate: dict[int, list[float]] = {}
        self.asked: dict[int, int] = {}
        self.drafted = self.accepted = self.calls = self.steps = 0

    # --- costs -----------------------------------------------------------------------------------------
    def _line(self) -> tuple[float, float]:
        """(seconds of a step's first row, seconds per further row)."""
        points = list(self.by_rows.items())
        if len(points) < 2:
            if points:
                base = points[0][1] - 0.0025 * (points[0][0] - 1)
            else:
                base = 0.085
            return max(1e-4, base), 0.0025
        count = len(points)
        mean_r = sum(r for r, _ in points) / count
        mean_t = sum(t for _, t in points) / count
        var = sum((r - mean_r) ** 2 for r, _ in points)
        if var > 0:
            slope = max(0.0005, sum((r - mean_r) * (t - mean_t) for r, t in points) / var)
        else:
            slope = 0.0025
        return max(1e-4, mean_t - slope * (mean_r - 1)), slope

    @property
    def c_row(self) -> float:
        return self._line()[1]

    def step_seconds(self, rows: int) -> float:
        if rows in self.by_rows:
            return self.by_rows[rows]
        first, slope = self._line()
        return first + slope * (rows - 1)

    def call_seconds(self, rows: int) -> float:
        if rows in self.call:
            return self.call[rows]
        if not self.call:
            return 0.015 + 0.001 * (rows - 1)
        near = min(self.call, key=lambda n: abs(n - rows))
        return max(1e-4, self.call[near] + 0.001 * (rows - near))

    # --- calibration -----------------------------------------------------------------------------------
    def p(self, confidence: float) -> float:
        b = _bin(confidence)
        return self.taken[b] / self.tried[b]

    def mean(self) -> float:
        return sum(self.taken) / sum(self.tried)

    # --- the rule --------------------------------------------------------------------------------------
    def start(self, running: int, sharers: int = 1) -> bool:
        """Draft in this step at all?"""
        self.asked[running] = self.asked.get(running, 0) + 1
        plain = running / self.step_seconds(running)
        seen = self.rate.get(running)
        if seen is not None and seen[1] >= self.TRUST and seen[0] < plain and self.asked[running] % self.PROBE:
            return False
        cost = self.call_seconds(sharers) + self.c_row * sharers
        return (running + sharers * self.mean()) / (self.step_seconds(running) + cost) > plain

    def more(self, q: float, expected: float, spent: float, running: int, sharers: int) -> bool:
        """One more draft for a request whose drafts so far all hold with chance `q`?"""
        cost = self.call_seconds(sharers) / max(1, sharers) + self.c_row
        return q * self.mean() / cost > (running + expected) / (self.step_seconds(running) + spent)

    # --- learning --------------------------------------------------------------------------------------
    def learn(self, confidences: Sequence[float], accepted: int) -> None:
        for i, confidence in enumerate(confidences[:accepted + 1]):
            b = _bin(confidence)
            self.tried[b] += 1
            self.taken[b] += i < accepted
        self.drafted += len(confidences)
        self.accepted += accepted

    def observe_call(self, seconds: float, rows: int = 1) -> None:
        old = self.call.get(rows)
        self.call[rows] = seconds if old is None else old + 0.1 * (seconds - old)
        self.calls += 1

    def observe_step(self, seconds: float, running: int, draft_rows: int, tokens: int | None = None,
                     draft_seconds: float = 0.0) -> None:
        rows = running + draft_rows
        old = self.by_rows.get(rows)
        self.by_rows[rows] = seconds if old is None else old + 0.1 * (seconds - old)
        if draft_seconds > 0 and tokens is not None:
            made = tokens / (seconds + draft_seconds)
            seen = self.rate.setdefault(running, [made, 0])
            seen[0] += 0.1 * (made - seen[0])
            seen[1] += 1
        self.steps += 1

    def summary(self) -> dict[str, Any]:
        first, slope = self._line()
        return {"drafted": self.drafted, "accepted": self.accepted, "draft_calls": self.calls,
                "acceptance_by_confidence": [round(a / b, 3) for a, b in zip(self.taken, self.tried)],
                "draft_call_ms_by_rows": {str(n): round(1000 * t, 1) for n, t in sorted(self.call.items())},
                "step_ms": round(1000 * first, 1), "row_ms": round(1000 * slope, 2),
                "tok_s_with_drafts_by_requests": {str(n): round(r[0], 1) for n, r in sorted(self.rate.items())}}


def _common(a: Sequence[int], b: Sequence[int]) -> int:
    """Length of the longest common prefix (64-token slices first, then token by token)."""
    if type(a) is not type(b):
        a, b = list(a), list(b)
    limit = min(len(a), len(b))
    i = 0
    while i + 64 <= limit and a[i:i + 64] == b[i:i + 64]:
        i += 64
    while i < limit and a[i] == b[i]:
        i += 1
    return i


class Drafter:
    """The draft model and its KV slots. `engine` implements `_decode_conf`, `eog`, `L`, `memory`, `seqs`."""

    def __init__(self, engine: Any, max_running: int = 2):
        self.e = engine
        self.max_running = max_running
        self.stop = DraftStop()
        self.held: dict[int, list[int]] = {slot: [] for slot in range(engine.seqs)}
        self.slot_of: dict[int, int] = {}
        self._pending: dict[int, tuple[int, list[float]]] = {}
        self.step_seconds = 0.0
        self.catchup_seconds = 0.0

    def _assign(self, key: int, context: Sequence[int]) -> int | None:
        taken = set(self.slot_of.values())
        free = [slot for slot in self.held if slot not in taken]
        if not free:
            return None
        slot = max(free, key=lambda s: _common(self.held[s], context))
        self.slot_of[key] = slot
        return slot

    def release(self, key: int) -> None:
        """The request ended; its slot keeps its cells for a later request with the same prefix."""
        self.slot_of.pop(key, None)
        self._pending.pop(key, None)

    def _call(self, rows: list[tuple[int, int, int, bool]], catchup: float = 0.0) -> list[tuple[int, float]]:
        began = time.perf_counter()
        out = self.e._decode_conf(rows)
        seconds = time.perf_counter() - began
        self.step_seconds += seconds
        self.catchup_seconds += seconds * catchup
        if len(out) == len(rows):
            self.stop.observe_call(seconds, len(rows))
        return out

    def _catch_up(self, key: int, context: Sequence[int]) -> list[tuple[int, int, int, bool]]:
        """Bring the key's slot up to `context`: trim cells past the shared prefix, read long catch-ups in
        CHUNK-token calls of their own; return the rows of the remainder (the last one wants logits)."""
        slot = self.slot_of[key]
        held = self.held[slot]
        shared = min(_common(held, context), len(context) - 1)  # the last token is always recomputed
        if len(held) > shared:
            if shared == 0 or not self.e.L.llama_memory_seq_rm(self.e.memory, slot, shared, -1):
                self.e.L.llama_memory_seq_rm(self.e.memory, slot, -1, -1)
                shared = 0
            del held[shared:]
        feed = context[shared:]
        while len(feed) > CHUNK:
            part, feed = feed[:CHUNK], feed[CHUNK:]
            self._call([(t, len(held) + j, slot, False) for j, t in enumerate(part)], catchup=1.0)
            held.extend(part)
        rows = [(t, len(held) + j, slot, j == len(feed) - 1) for j, t in enumerate(feed)]
        held.extend(feed)
        return rows

    def draft(self, wants: dict[int, tuple[Sequence[int], int]], running: int) -> dict[int, list[int]]:
        """Drafts for the requests in `wants` (key -> (tokens so far, room for drafts)), as many as the rule
        allows; {} where it gives none. `running` is the number of requests in the step."""
        self.step_seconds = self.catchup_seconds = 0.0
        if running > self.max_running:
            return {}
        keys = [key for key in wants if key in self.slot_of or self._assign(key, wants[key][0]) is not None]
        if not keys or not self.stop.start(running, len(keys)):
            return {}
        rows: list[tuple[int, int, int, bool]] = []
        for key in keys:
            rows += self._catch_up(key, wants[key][0])
        picks = self._call(rows, catchup=(len(rows) - len(keys)) / max(1, len(rows)))
        nxt = {key: picks[i] for i, key in enumerate(keys)}
        drafts: dict[int, list[int]] = {key: [] for key in keys}
        confs: dict[int, list[float]] = {key: [] for key in keys}
        chance = {key: 1.0 for key in keys}
        expected, spent, going = 0.0, self.step_seconds, list(keys)
        while going:
            again = []
            for key in going:
                token, confidence = nxt[key]
                drafts[key].append(token)
                confs[key].append(confidence)
                chance[key] *= self.stop.p(confidence)
                expected += chance[key]
                if len(drafts[key]) < wants[key][1] and not self.e.eog(token):
                    again.append(key)
            going = [key for key in again if self.stop.more(chance[key], expected, spent, running, len(again))]
            if not going:
                break
            rows = []
            for key in going:
                slot = self.slot_of[key]
                rows.append((drafts[key][-1], len(self.held[slot]), slot, True))
                self.held[slot].append(drafts[key][-1])
            picks = self._call(rows)
            spent = self.step_seconds + self.stop.c_row * sum(len(drafts[k]) for k in keys)
            for key, pick in zip(going, picks):
                nxt[key] = pick
        for key in keys:
            self._pending[key] = (len(wants[key][0]), confs[key])
        return {key: drafts[key] for key in keys}

    def settle(self, key: int, used: int, accepted: int) -> None:
        """The target verified the first `used` drafts of the request and kept `accepted` of them."""
        pending = self._pending.pop(key, None)
        slot = self.slot_of.get(key)
        if pending is None or slot is None:
            return
        before, confidences = pending
        self.stop.learn(confidences[:used], accepted)
        held = self.held[slot]
        keep = before + min(accepted, max(0, len(held) - before))
        if len(held) > keep:
            self.e.L.llama_memory_seq_rm(self.e.memory, slot, keep, -1)
            del held[keep:]

    def end_step(self, seconds: float, running: int, draft_rows: int, tokens: int) -> None:
        """The step the drafts were for took `seconds` and made `tokens` tokens."""
        drafting = max(1e-6, self.step_seconds - self.catchup_seconds) if draft_rows else 0.0
        self.stop.observe_step(seconds, running, draft_rows, tokens, drafting)
        self.step_seconds = self.catchup_seconds = 0.0

    def summary(self) -> dict[str, Any]:
        return {"slots": len(self.held), "max_running": self.max_running, **self.stop.summary()}

    def close(self) -> None:
        close = getattr(self.e, "close", None)
        if close is not None:
            close()


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
