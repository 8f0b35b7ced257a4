"""TEST INFRASTRUCTURE ONLY: the speculative round on the CPU -- the oracle port of the device round, used
as the timed CPU baseline (`bench.py` cpu_baseline and --impl reference) and as a parity checker.

The round is the device round's (ironmule_b200/csrc/spec.cu): draft pass 0 over the last two committed
tokens, draft passes 1..k-1 over one draft each, one verify forward of the target over k+1 rows, greedy
acceptance (IronMule ironmule/speculation.py:103-108), append -- the host loop of
ironmule/ggml_engine.py:1155-1343 with a draft model (ironmule/draft_model.py:203-274) at a fixed k.
"""
from __future__ import annotations

import numpy as np

from . import bf16
from .accept import greedy_accept, row_stats
from .model import OracleModel


class CpuSpecDecoder:
    def __init__(self, target: OracleModel, draft: OracleModel, k: int = 4, slots: int = 1024):
        self.target, self.draft, self.k, self.slots = target, draft, k, slots
        self.hist: list[int] = []
        self.margins: list[float] = []  # per committed token: top-2 logit margin of the verify row that chose it
        self.tops: list[float] = []     # ... and that row's top logit
        self.rounds = self.accepted = 0

    def start(self, prompt: list[int]) -> None:
        self.target.reset(self.slots)
        self.draft.reset(self.slots)
        self.hist = list(prompt)
        self.margins, self.tops = [], []
        if len(prompt) > 1:
            pos = list(range(len(prompt) - 1))
            self.target.forward(prompt[:-1], pos, logits=False)
            self.draft.forward(prompt[:-1], pos, logits=False)
        self.rounds = self.accepted = 0

    def round(self) -> list[int]:
        n, k = len(self.hist), self.k
        logits = self.draft.forward([self.hist[n - 2], self.hist[n - 1]], [n - 2, n - 1])
        drafts = [int(row_stats(logits[-1:])[0][0])]
        for i in range(1, k):
            logits = self.draft.forward([drafts[-1]], [n - 1 + i])
            drafts.append(int(row_stats(logits)[0][0]))
        vlog = self.target.forward([self.hist[n - 1]] + drafts, list(range(n - 1, n + k)))
        picks = row_stats(vlog)[0].tolist()
        kept = greedy_accept(drafts, picks)
        self.margins.extend(top2_margin(vlog[i]) for i in range(len(kept)))
        self.tops.extend(float(bf16.to_f32(vlog[i]).max()) for i in range(len(kept)))
        self.hist.extend(kept)
        self.rounds += 1
        self.accepted += len(kept) - 1
        return kept


def top2_margin(row_bits: np.ndarray) -> float:
    """The gap between the largest and the second-largest logit of a row (0 for a tie at the top)."""
    f = bf16.to_f32(row_bits).astype(np.float64)
    top2 = np.partition(f, -2)[-2:]
    return float(top2[1] - top2[0])


def random_model(cfg, seed: int = 0, slots: int = 256, fast: bool = True) -> OracleModel:
    """A CPU model of `cfg`'s shapes with random 4-bit codes, scales and biases (for timing the CPU baseline;
    the parity tests use weights copied from the device instead)."""
    from .model import HostLayer

    rng = np.random.default_rng(seed)

    def lin(n, k):
        wq = rng.integers(0, 2 ** 32, size=(n, k // 8), dtype=np.uint32)
        scale = np.abs(rng.normal(0, 0.004, (n, k // 64))).astype(np.float32) + 1e-4
        from . import bf16
        return wq, bf16.from_f32(scale), bf16.from_f32(-7.5 * scale)

    def vec(n, base):
        from . import bf16
        return bf16.from_f32((base + 0.02 * rng.normal(0, 1, n)).astype(np.float32))

    base = 0.0 if cfg.family == "gemma3" else 1.0
    layers = [HostLayer(lin(cfg.qkv_rows, cfg.hidden), lin(cfg.hidden, cfg.heads * cfg.head_dim),
                        lin(2 * cfg.inter, cfg.hidden), lin(cfg.hidden, cfg.inter), vec(cfg.hidden, base),
                        vec(cfg.hidden, base), vec(cfg.head_dim, base), vec(cfg.head_dim, base))
              for _ in range(cfg.layers)]
    d = cfg.head_dim
    idx = np.arange(d // 2, dtype=np.float64)
    model = OracleModel(cfg, lin(cfg.vocab, cfg.hidden), layers, vec(cfg.hidden, base),
                        (cfg.rope_theta ** (-2 * idx / d)).astype(np.float32),
                        (cfg.rope_local_theta ** (-2 * idx / d)).astype(np.float32), fast=fast)
    model.reset(slots)
    return model
