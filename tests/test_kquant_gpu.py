"""The GGUF k-quant matmul on the B200 (im_kq_gemv / im_kq_mul_mat) against the CPU oracle's restatement of its
arithmetic (oracle/kquant_oracle.c): bit for bit for Q4_K and Q6_K at 1-32 tokens (Q4_K from 3 tokens runs on int8
tensor-core MMA, the rest on dp4a: the same bits), ragged row counts and K from one block up; a token's results
alone equal its results in a batch; the relative L2 error against float64 within the reference's bound (1.25 x 6e-3, ironmule/kernel_gen.py:615, 1001, 1023); the hook's refusals for what it does not
serve (ironmule/kernel_gen.py:803-806); a Q4_K matrix read from a GGUF file."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from ironmule_b200 import _lib, gguf, kernels
from oracle import kquant as kq

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def run(kind, n, k, b, seed, hook=False):
    w = kq.random_blocks(kind, n * k // 256, seed=seed)
    x = np.random.default_rng(seed + 1).normal(0, 1, (b, k)).astype(np.float32)
    wd = torch.from_numpy(w.reshape(-1)).cuda()
    xd = torch.from_numpy(x).cuda()
    if hook:
        rc, y = kernels.kq_mul_mat(kind, wd, xd, n)
        assert rc == 0
    else:
        y = kernels.kq_gemv(kind, wd, xd, n)
    return w, x, y.cpu().numpy()


@pytest.mark.parametrize("kind", [kq.Q4_K, kq.Q6_K])
@pytest.mark.parametrize("n,k,b", [(1, 256, 1), (7, 512, 2), (264, 2048, 3), (100, 1280, 5), (64, 768, 8),
                                   (33, 2560, 13), (300, 1024, 16), (17, 4096, 32), (7, 256, 6), (1, 1792, 4),
                                   (529, 2560, 5)])
def test_bit_exact_against_the_oracle(cuda, kind, n, k, b):
    w, x, y = run(kind, n, k, b, seed=n + k + b)
    want = kq.gemv(kind, w, n, x)
    assert np.array_equal(y.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("kind", [kq.Q4_K, kq.Q6_K])
def test_hook_entry_and_token_independence(cuda, kind):
    n, k = 520, 2560
    w, x, y = run(kind, n, k, 32, seed=5, hook=True)
    assert np.array_equal(y.view(np.uint32), kq.gemv(kind, w, n, x).view(np.uint32))
    wd = torch.from_numpy(w.reshape(-1)).cuda()
    for t in (0, 9, 31):
        one = kernels.kq_gemv(kind, wd, torch.from_numpy(x[t:t + 1]).cuda(), n).cpu().numpy()
        assert np.array_equal(one.view(np.uint32), y[t:t + 1].view(np.uint32)), t


@pytest.mark.parametrize("kind", [kq.Q4_K, kq.Q6_K])
def test_error_within_the_reference_bound(cuda, kind):
    n, k = 512, 4096
    w, x, y = run(kind, n, k, 4, seed=11)
    ref = kq.ref64(kind, w, n, x)
    assert np.sqrt(np.sum((y - ref) ** 2) / np.sum(ref ** 2)) <= 1.25 * 6e-3


def test_refusals(cuda):
    w = torch.from_numpy(kq.random_blocks(kq.Q4_K, 8, seed=1).reshape(-1)).cuda()
    x = torch.zeros((1, 2048), dtype=torch.float32, device="cuda")
    y = torch.zeros((1, 1), dtype=torch.float32, device="cuda")
    lib = _lib.load()
    s = torch.cuda.current_stream().cuda_stream
    assert lib.im_kq_mul_mat(2, w.data_ptr(), x.data_ptr(), y.data_ptr(), 1, 2048, 1, s) == _lib.IM_UNSUPPORTED
    assert lib.im_kq_mul_mat(12, w.data_ptr(), x.data_ptr(), y.data_ptr(), 1, 2000, 1, s) == _lib.IM_UNSUPPORTED
    assert lib.im_kq_mul_mat(12, w.data_ptr(), x.data_ptr(), y.data_ptr(), 1, 2048, 33, s) == _lib.IM_UNSUPPORTED
    assert lib.im_kq_mul_mat(12, w.data_ptr() + 2, x.data_ptr(), y.data_ptr(), 1, 2048, 1, s) == _lib.IM_INVALID
    big = 1 << 20  # K x tokens beyond the hook's scratch
    assert lib.im_kq_mul_mat(12, w.data_ptr(), x.data_ptr(), y.data_ptr(), 1, big, 32, s) == _lib.IM_UNSUPPORTED
    with pytest.raises(_lib.KernelUnsupported):
        kernels.kq_gemv(12, w, torch.zeros((33, 2048), dtype=torch.float32, device="cuda"), 1)


def test_gguf_matrix_on_the_device(cuda):
    f = gguf.GGUFFile(GOLDEN / "tiny.gguf")
    for name in ("blk.0.ffn_down.weight", "output.weight"):
        lin = gguf.kquant_linear(f, name)
        x = np.random.default_rng(2).normal(0, 1, (3, lin.k)).astype(np.float32)
        y = lin(torch.from_numpy(x).cuda()).cpu().numpy()
        want = kq.gemv(lin.kind, np.asarray(f.raw(name)), lin.n, x)
        assert np.array_equal(y.view(np.uint32), want.view(np.uint32)), name


@pytest.mark.parametrize("kind", [kq.Q4_K, kq.Q6_K])
def test_unaligned_activations(cuda, kind):
    """Activations only 4-byte aligned (a view one float into a buffer) give the same bits."""
    n, k, b = 96, 1024, 3
    w = kq.random_blocks(kind, n * k // 256, seed=31)
    x = np.random.default_rng(32).normal(0, 1, (b, k)).astype(np.float32)
    buf = torch.zeros(b * k + 1, dtype=torch.float32, device="cuda")
    xd = buf[1:].view(b, k)
    xd.copy_(torch.from_numpy(x))
    assert xd.data_ptr() % 16 == 4
    y = kernels.kq_gemv(kind, torch.from_numpy(w.reshape(-1)).cuda(), xd, n).cpu().numpy()
    assert np.array_equal(y.view(np.uint32), kq.gemv(kind, w, n, x).view(np.uint32))
