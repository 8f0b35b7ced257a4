"""Device argmax / top-1 probability and greedy verification against numpy and the host `accept`
(ironmule/speculation.py:103-108, ironmule/ggml_engine.py:669-683)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from ironmule_b200 import kernels
from ironmule_b200 import speculation as sp
from oracle import bf16

from .gpu_util import bf16_bits_to_torch

pytestmark = pytest.mark.gpu


def np_stats(rows_f32: np.ndarray):
    idx = rows_f32.argmax(axis=1)  # numpy: first index of the max
    mx = rows_f32.max(axis=1, keepdims=True)
    conf = 1.0 / np.exp(rows_f32.astype(np.float64) - mx).sum(axis=1)
    return idx, conf


@pytest.mark.parametrize("rows,v", [(5, 151936), (1, 262144), (3, 1000), (7, 37), (160, 151936)])
def test_argmax_and_confidence(cuda, rows, v):
    rng = np.random.default_rng(rows + v)
    logits = bf16.from_f32((rng.normal(0, 3, (rows, v))).astype(np.float32))
    t = bf16_bits_to_torch(logits, cuda)
    idx, conf = kernels.argmax_rows(t, with_conf=True)
    want_idx, want_conf = np_stats(bf16.to_f32(logits))
    assert np.array_equal(idx.cpu().numpy(), want_idx)
    assert np.allclose(conf.cpu().numpy(), want_conf, rtol=1e-4)


def test_ties_take_the_lowest_index(cuda):
    v = 151936
    row = np.full((4, v), -1.0, dtype=np.float32)
    row[0, [5, 90000, 151935]] = 7.0
    row[1, [151935, 151934]] = 2.0
    row[2, :] = 0.5                      # all equal
    row[3, [4096, 4095, 8191]] = 3.0     # across chunk boundaries
    t = bf16_bits_to_torch(bf16.from_f32(row), cuda)
    idx, _ = kernels.argmax_rows(t)
    assert idx.cpu().tolist() == [5, 151934, 0, 4095]


def test_misaligned_rows_take_the_scalar_path(cuda):
    rng = np.random.default_rng(1)
    v = 1001
    logits = bf16.from_f32(rng.normal(0, 1, (6, v)).astype(np.float32))
    t = bf16_bits_to_torch(logits, cuda)
    idx, _ = kernels.argmax_rows(t)  # rows of 1001 bf16 are not 16-byte aligned
    assert np.array_equal(idx.cpu().numpy(), bf16.to_f32(logits).argmax(axis=1))


@pytest.mark.parametrize("b,k", [(1, 4), (32, 4), (8, 15), (3, 0)])
def test_verify_greedy_equals_host_accept(cuda, b, k):
    rng = np.random.default_rng(b * 100 + k)
    v = 5000
    logits = bf16.from_f32(rng.normal(0, 2, (b * (k + 1), v)).astype(np.float32))
    picks = bf16.to_f32(logits).argmax(axis=1).reshape(b, k + 1)
    drafts = np.where(rng.random((b, k)) < 0.7, picks[:, :k], rng.integers(0, v, (b, k))).astype(np.int32)
    for i in range(0, b, 3):
        drafts[i] = picks[i, :k]        # some sequences accept everything
    tokens, count = kernels.verify_greedy(bf16_bits_to_torch(logits, cuda), torch.from_numpy(drafts).to(cuda))
    tokens, count = tokens.cpu().numpy(), count.cpu().numpy()
    for i in range(b):
        want = sp.accept(list(drafts[i]), list(picks[i]))
        assert count[i] == len(want)
        assert list(tokens[i, :count[i]]) == want
        assert np.all(tokens[i, count[i]:] == -1)


def test_workspace_is_reusable_across_calls(cuda):
    rng = np.random.default_rng(2)
    for _ in range(3):
        logits = bf16.from_f32(rng.normal(0, 1, (5, 151936)).astype(np.float32))
        idx, _ = kernels.argmax_rows(bf16_bits_to_torch(logits, cuda))
        assert np.array_equal(idx.cpu().numpy(), bf16.to_f32(logits).argmax(axis=1))
