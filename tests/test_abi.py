"""The C ABI without a GPU: the library loads, exports every function include/imspec.h declares, and rejects
bad arguments (null pointers, bad sizes, misalignment) with a status and a message, launching nothing."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from ironmule_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "imspec.h"


def declared() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b((?:im|ironmule_kg)_[a-z0-9_]+)\s*\(", text)))


def test_every_declared_symbol_is_exported_and_typed():
    lib = _lib.load()
    names = declared()
    assert len(names) >= 9 and "ironmule_kg_mul_mat" in names
    for name in names:
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_abi_version():
    assert _lib.load().im_abi_version() == _lib.ABI_VERSION == 1


def _status(name, *args):
    lib = _lib.load()
    return getattr(lib, name)(*args), lib.im_last_error().decode()


def test_qgemm_rejects_bad_arguments_without_launching():
    rc, msg = _status("im_qgemm_w4g64", None, None, None, None, None, 1, 16, 64, None)
    assert rc == _lib.IM_INVALID and "null" in msg
    rc, msg = _status("im_qgemm_w4g64", 16, 16, 16, 16, 16, 1, 16, 100, None)
    assert rc == _lib.IM_UNSUPPORTED and "64" in msg
    rc, msg = _status("im_qgemm_w4g64", 16, 16, 16, 16, 16, 1, 0, 64, None)
    assert rc == _lib.IM_INVALID
    rc, msg = _status("im_qgemm_w4g64", 8, 16, 16, 16, 16, 1, 16, 64, None)  # w not 16-byte aligned
    assert rc == _lib.IM_INVALID and "aligned" in msg
    rc, msg = _status("im_qgemm_w4g64", 16, 16, 16, 16, 16, 33, 16, 64, None)
    assert rc == _lib.IM_UNSUPPORTED and "M <= 32" in msg
    rc, msg = _status("im_qgemm_w4g64_ex", 16, 16, 16, 16, 16, None, 9, 16, 64, 0, _lib.QGEMM_FMA, None, 0, None)
    assert rc == _lib.IM_UNSUPPORTED and "M <= 8" in msg
    rc, msg = _status("im_qgemm_w4g64_ex", 16, 16, 16, 16, 16, None, 1, 16, 64, _lib.EPI_RESIDUAL, 0, None, 0, None)
    assert rc == _lib.IM_INVALID and "residual" in msg
    rc, msg = _status("im_qgemm_w4g64_ex", 16, 16, 16, 16, 16, None, 1, 48, 64, _lib.EPI_SWIGLU, 0, None, 0, None)
    assert rc == _lib.IM_INVALID and "32" in msg
    # M == 0 is a no-op that succeeds
    rc, msg = _status("im_qgemm_w4g64", None, None, None, None, None, 0, 16, 64, None)
    assert rc == _lib.IM_OK and msg == ""


def test_workspace_sizes():
    lib = _lib.load()
    assert lib.im_qgemm_workspace_bytes(5, 15360, 3840) >= 0
    assert lib.im_qgemm_workspace_bytes(5, 2560, 9728) > 0      # small N, long K: CTAs split K
    assert lib.im_qgemm_workspace_bytes(0, 16, 64) == 0
    assert lib.im_argmax_workspace_bytes(5, 151936) > 256


def test_argmax_rejects_bad_arguments():
    rc, msg = _status("im_argmax_rows", 16, 0, 10, 10, 16, 1, None, 256, 1 << 20, None)
    assert rc == _lib.IM_INVALID
    rc, msg = _status("im_argmax_rows", 16, 2, 10, 10, 16, 1, None, 256, 8, None)
    assert rc == _lib.IM_INVALID and "workspace" in msg
    rc, msg = _status("im_verify_greedy", 16, 1, 4, 10, 10, None, 4, 16, 16, None, 256, 1 << 20, None)
    assert rc == _lib.IM_INVALID


def test_errors_raise_typed_exceptions():
    with pytest.raises(_lib.KernelUnsupported):
        _lib.call("im_qgemm_w4g64", 16, 16, 16, 16, 16, 1, 16, 100, None)
    with pytest.raises(_lib.KernelError):
        _lib.call("im_qgemm_w4g64", None, None, None, None, None, 1, 16, 64, None)


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(_lib.KernelLibraryMissing):
        _lib.load(tmp_path / "libimspec.so")


def test_kquant_rejects_bad_arguments_without_launching():
    rc, msg = _status("im_kq_mul_mat", 2, None, None, None, 1, 256, 1, None)
    assert rc == _lib.IM_UNSUPPORTED and "type" in msg
    rc, msg = _status("ironmule_kg_mul_mat", 12, None, None, None, 1, 300, 1, None)
    assert rc == _lib.IM_UNSUPPORTED
    rc, msg = _status("im_kq_gemv", 12, None, None, None, 1, 256, 1, None, 0, None)
    assert rc == _lib.IM_INVALID and "null" in msg
    assert _lib.load().im_kq_workspace_bytes(2560, 4) >= 4 * 2560 + 2 * 4 * 80 * 4
