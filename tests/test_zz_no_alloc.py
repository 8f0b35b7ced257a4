"""The qGEMM entry point for callers that cannot allocate device memory (im_qgemm_w4g64_noalloc).

Such callers -- an engine that hands out all device memory from its own pool, a plugin that may not call
cudaMalloc or synchronise the device on its decode path -- pass only inputs and outputs; the entry point keeps
the split-K scratch in a static device array. This file is collected last on purpose: it checks the entry point
through the C ABI against the workspace entry point, twice in a row (the shared array must come back clean), and
that a shape too large for the static array is refused without launching."""
from __future__ import annotations

import subprocess
import sys
import textwrap
from pathlib import Path

import numpy as np
import pytest
import torch

from ironmule_b200 import _lib, kernels

from .gpu_util import MAX_REL, MEAN_REL, case, rel_errors, to_device, torch_to_bf16_bits

pytestmark = pytest.mark.gpu


def noalloc(x, w, s, b):
    m, k = x.shape
    y = torch.empty((m, w.shape[0]), dtype=torch.bfloat16, device=x.device)
    _lib.call("im_qgemm_w4g64_noalloc", w.data_ptr(), s.data_ptr(), b.data_ptr(), x.data_ptr(), y.data_ptr(), m,
              w.shape[0], k, torch.cuda.current_stream(x.device).cuda_stream)
    return y


@pytest.mark.parametrize("n,k,m", [(2560, 9728, 5), (15360, 3840, 5), (1024, 3072, 1)])
def test_noalloc_matches_the_workspace_entry_point_twice(cuda, n, k, m):
    wq, s, b, x = case(n, k, m, seed=n + k)
    w_t, s_t, b_t, x_t = to_device(wq, s, b, x, cuda)
    want = torch_to_bf16_bits(kernels.qgemm(x_t, w_t, s_t, b_t, split_k=True))
    for _ in range(2):
        got = torch_to_bf16_bits(noalloc(x_t, w_t, s_t, b_t))
        torch.cuda.synchronize()
        mx, mean = rel_errors(got, want)
        assert mx <= MAX_REL and mean <= MEAN_REL
        assert np.array_equal(got, want)  # the same split plan: the same bits


def test_noalloc_refuses_shapes_beyond_its_scratch(cuda):
    lib = _lib.load()
    assert lib.im_qgemm_noalloc_capacity() == 8 << 20
    assert lib.im_qgemm_workspace_bytes(1, 35200, 1024) > lib.im_qgemm_noalloc_capacity()
    x = torch.zeros((1, 1024), dtype=torch.bfloat16, device=cuda)
    w = torch.zeros((35200, 128), dtype=torch.int32, device=cuda)
    sb = torch.zeros((35200, 16), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(_lib.KernelUnsupported, match="static scratch"):
        noalloc(x, w, sb, sb)


FIRST_CALL_ON_A_SIDE_STREAM = textwrap.dedent("""
    import sys
    import numpy as np
    import torch
    sys.path.insert(0, sys.argv[1])
    from ironmule_b200 import _lib, kernels
    from tests.gpu_util import case, to_device, torch_to_bf16_bits
    dev = torch.device("cuda:0")
    wq, s, b, x = case(2560, 9728, 5, seed=7)
    w_t, s_t, b_t, x_t = to_device(wq, s, b, x, dev)
    want = torch_to_bf16_bits(kernels.qgemm(x_t, w_t, s_t, b_t, split_k=True))
    side = torch.cuda.Stream(dev)   # a non-blocking stream: not ordered behind the legacy default stream
    side.wait_stream(torch.cuda.current_stream(dev))
    outs = []
    with torch.cuda.stream(side):
        for _ in range(2):
            y = torch.empty((5, 2560), dtype=torch.bfloat16, device=dev)
            _lib.call("im_qgemm_w4g64_noalloc", w_t.data_ptr(), s_t.data_ptr(), b_t.data_ptr(), x_t.data_ptr(),
                      y.data_ptr(), 5, 2560, 9728, side.cuda_stream)
            outs.append(y)
    side.synchronize()
    for y in outs:
        assert np.array_equal(torch_to_bf16_bits(y), want), "no-alloc call on a side stream changed the bits"
    print("ok")
""")


def test_noalloc_first_call_on_a_side_stream(cuda):
    """The first call on a device zeroes the shared counters; on a non-blocking stream that zeroing must still
    come before the kernel. A fresh process makes this call the device's first."""
    root = Path(__file__).resolve().parents[1]
    run = subprocess.run([sys.executable, "-c", FIRST_CALL_ON_A_SIDE_STREAM, str(root)], capture_output=True,
                         text=True, timeout=300, cwd=root)
    assert run.returncode == 0 and run.stdout.strip().endswith("ok"), run.stdout + run.stderr
