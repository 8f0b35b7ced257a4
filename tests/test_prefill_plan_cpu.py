"""The packed prefill's plan on the CPU: every prompt is cut into exactly the chunks a one-by-one prefill cuts
(in order, `step` tokens each, the last shorter), each forward stays within the row budget and holds at most one
chunk per prompt, and nothing is left out."""
from __future__ import annotations

import random

import pytest

from ironmule_b200.engine import prefill_plan


@pytest.mark.parametrize("seed", range(40))
def test_plan_covers_each_prompt_in_its_own_chunks(seed):
    rng = random.Random(seed)
    lengths = [rng.randint(0, 600) for _ in range(rng.randint(1, 12))]
    step = rng.choice([32, 64, 128, 256])  # 32: the fused attention's chunk; wider chunks go through two kernels
    budget = rng.choice([b for b in (32, 64, 96, 160, 256, 320) if b >= step])
    plan = prefill_plan(lengths, step, budget)
    seen = {i: [] for i in range(len(lengths))}
    for forward in plan:
        assert sum(c for _, _, c in forward) <= budget
        assert len({i for i, _, _ in forward}) == len(forward)
        for i, off, c in forward:
            seen[i].append((off, c))
    for i, n in enumerate(lengths):
        assert seen[i] == [(o, min(step, n - o)) for o in range(0, n, step)], i


def test_bad_arguments():
    with pytest.raises(ValueError):
        prefill_plan([10], 0, 32)
    with pytest.raises(ValueError):
        prefill_plan([10], 32, 16)
    assert prefill_plan([], 32, 64) == [] and prefill_plan([0, 0], 32, 64) == []
