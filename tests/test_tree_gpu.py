"""Tree speculation on the device: top-k against numpy, the tree walk against a Python walk, and the decoder's
invariant -- a node sees the committed prefix plus its own path and every kernel is row-invariant, so tree
speculation returns exactly the tokens of plain greedy decoding, for several tree shapes; with the target as
its own draft every round accepts a full-depth path."""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from ironmule_b200 import engine, kernels
from oracle import bf16

from .gpu_util import bf16_bits_to_torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,v,k", [(1, 151936, 4), (8, 1000, 2), (3, 5000, 8)])
def test_topk_matches_numpy(cuda, rows, v, k):
    rng = np.random.default_rng(rows + k)
    x = bf16.from_f32(rng.normal(0, 1, (rows, v)).astype(np.float32))
    x[0, 17] = x[0, 4000 % v] = bf16.from_f32(np.array([9.0], dtype=np.float32))[0]  # a tie at the top
    got = kernels.topk_rows(bf16_bits_to_torch(x, cuda), k).cpu().numpy()
    f = bf16.to_f32(x)
    for r in range(rows):
        want = np.lexsort((np.arange(v), -f[r]))[:k]  # value descending, then index ascending
        assert got[r].tolist() == want.tolist(), r


def walk(argmax, tok, branch):
    counts = [math.prod(branch[:i + 1]) for i in range(len(branch))]
    first = [sum(counts[:i]) for i in range(len(branch))]
    row, out, nodes = 0, [], []
    child0, nchild = 0, branch[0]
    for depth in range(len(branch)):
        want = argmax[row]
        hit = next((child0 + c for c in range(nchild) if tok[1 + child0 + c] == want), None)
        if hit is None:
            break
        out.append(want)
        nodes.append(hit)
        row = 1 + hit
        if depth + 1 < len(branch):
            nchild = branch[depth + 1]
            child0 = first[depth + 1] + (hit - first[depth]) * nchild
    return out + [argmax[row]], nodes


def test_tree_accept_matches_a_python_walk(cuda):
    branch = (4, 2, 2)
    rng = np.random.default_rng(0)
    rows = 1 + 4 + 8 + 16
    for trial in range(30):
        tok = rng.integers(0, 6, rows).astype(np.int32)
        argmax = rng.integers(0, 6, rows).astype(np.int32)
        out_t = torch.zeros((1, 4), dtype=torch.int32, device=cuda)
        out_c = torch.zeros((1,), dtype=torch.int32, device=cuda)
        acc = torch.zeros((3,), dtype=torch.int32, device=cuda)
        kernels.tree_accept(torch.from_numpy(argmax).to(cuda), torch.from_numpy(tok).to(cuda), 1, branch, out_t, out_c,
                            acc)
        want, nodes = walk(argmax, tok, branch)
        c = int(out_c.item())
        assert out_t[0, :c].tolist() == want, trial
        assert acc.tolist() == nodes + [-1] * (3 - len(nodes)), trial


def tiny(name, seed):
    return engine.QuantModel(engine.PRESETS[name], "cuda", seed=seed, sigma=0.08, max_ctx=256)


@pytest.mark.parametrize("branch", [(4, 2, 2), (2, 2), (3,)])
def test_tree_speculation_changes_no_answer(cuda, branch):
    target, draft, solo = tiny("tiny-target", 1), tiny("tiny-draft", 2), tiny("tiny-target", 1)
    prompt = torch.randint(0, 1000, (21,), generator=torch.Generator().manual_seed(9)).to(torch.int32).to(cuda)
    plain = engine.greedy_decode(solo, prompt, 30)
    dec = engine.TreeDecoder(target, draft, branch=branch)
    dec.start([prompt], max_new=30)
    dec.round()
    dec.capture()
    while not dec.done():
        dec.run_rounds(2)
    assert dec.generated(0, prompt.numel()) == plain


def test_identical_draft_accepts_full_depth(cuda):
    target, draft = tiny("tiny-target", 1), tiny("tiny-target", 1)
    prompt = torch.arange(5, 30, dtype=torch.int32, device=cuda)
    dec = engine.TreeDecoder(target, draft, branch=(4, 2, 2))
    dec.start([prompt], max_new=24)
    dec.run_rounds(5)
    st = dec.read_stats()
    assert st.rounds == 5 and st.accepted == 15 and st.tokens == 20
    solo = tiny("tiny-target", 1)
    assert dec.generated(0, prompt.numel()) == engine.greedy_decode(solo, prompt, 20)


@pytest.mark.parametrize("branch", [(4, 2, 2), (2, 3)])
def test_batched_trees_change_no_answer(cuda, branch):
    """Several sequences of different lengths in one tree round: each level's rows gathered across the
    sequences, the verify forward over every sequence's tree; each sequence still returns its own greedy
    tokens."""
    b = 3
    target = engine.QuantModel(engine.PRESETS["tiny-target"], "cuda", seed=1, sigma=0.08, max_ctx=256, max_seqs=b,
                               max_rows=32 * b, max_logit_rows=32 * b)
    draft = engine.QuantModel(engine.PRESETS["tiny-draft"], "cuda", seed=2, sigma=0.08, max_ctx=256, max_seqs=b,
                              max_rows=32 * b, max_logit_rows=32 * b)
    gen = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, 1000, (n,), generator=gen).to(torch.int32).to(cuda) for n in (21, 9, 40)]
    dec = engine.TreeDecoder(target, draft, branch=branch, batch=b)
    dec.start(prompts, max_new=30)
    dec.round()
    dec.capture()
    while not dec.done():
        dec.run_rounds(2)
    for s, p in enumerate(prompts):
        solo = tiny("tiny-target", 1)
        assert dec.generated(s, p.numel()) == engine.greedy_decode(solo, p, 30), s
