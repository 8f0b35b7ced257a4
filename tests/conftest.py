"""Test configuration: the `gpu` marker (tests that need a B200), repo root on sys.path, and shared helpers.

`python -m pytest tests -m "not gpu"` runs on any machine (oracle pins, host parity, ABI checks);
`python -m pytest tests -m gpu` runs the kernels against the oracle on a B200.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a) and libimspec.so")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device; run it with -m gpu on a B200")
    major, _ = torch.cuda.get_device_capability()
    if major != 10:
        pytest.fail(f"libimspec is built for sm_100a; this device is sm_{major}x")
    return torch.device("cuda:0")
