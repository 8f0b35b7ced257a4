"""Loads libimspec.so (the sm_100a kernels) and declares its C ABI for ctypes.

There is no CPU fallback: if the library is missing or cannot load, every kernel call raises
`KernelLibraryMissing` naming the build command. The declarations mirror include/imspec.h.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libimspec.so"

IM_OK, IM_UNSUPPORTED, IM_INVALID, IM_CUDA_ERROR = 0, 1, 2, 3
EPI_STORE, EPI_RESIDUAL, EPI_SWIGLU, EPI_GEGLU = 0, 1, 2, 3
QGEMM_AUTO, QGEMM_MMA, QGEMM_FMA = 0, 1, 2
ABI_VERSION = 1

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_SZ = ctypes.c_size_t
_INT = ctypes.c_int

# name -> (restype, argtypes); every symbol include/imspec.h declares.
SIGNATURES: dict[str, tuple] = {
    "im_abi_version": (_INT, []),
    "im_last_error": (ctypes.c_char_p, []),
    "im_qgemm_w4g64": (_INT, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _P]),
    "im_qgemm_w4g64_ex": (_INT, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _INT, _INT, _P, _SZ, _P]),
    "im_qgemm_workspace_bytes": (_SZ, [_I64, _I64, _I64]),
    "im_qgemm_w4g64_noalloc": (_INT, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _P]),
    "im_qgemm_noalloc_capacity": (_SZ, []),
    "im_qgemm_set_splits": (_INT, [_INT]),
    "im_qgemm_packed_bytes": (_SZ, [_I64, _I64]),
    "im_qgemm_pack_w4g64": (_INT, [_P, _P, _P, _I64, _I64, _P, _P]),
    "im_qgemm_packed_workspace_bytes": (_SZ, [_I64, _I64, _I64]),
    "im_qgemm_packed_tune": (_INT, [_INT, _INT, _INT]),
    "im_qgemm_packed_status": (_INT, [_P]),
    "im_qgemm_packed_path": (_INT, [_INT]),
    "im_qgemm_packed_cluster": (_INT, [_INT]),
    "im_set_launch_overlap": (_INT, [_INT]),
    "im_rmsnorm_residual": (_INT, [_P, _P, _P, _I64, _I64, ctypes.c_float, _INT, _P, _P]),
    "im_topk_workspace_bytes": (_SZ, [_I64, _I64, _I64]),
    "im_topk_rows": (_INT, [_P, _I64, _I64, _I64, _I64, _P, _I64, _P, _SZ, _P]),
    "im_tree_prepare": (_INT, [_P, _I64, _P, _I64, _P, _I64, _I64, _P, _P, _P, _P, _P, _P, _P, _P]),
    "im_tree_accept": (_INT, [_P, _P, _I64, _P, _I64, _P, _P, _P, _P]),
    "im_tree_compact": (_INT, [_P, _P, _I64, _I64, _P, _I64, _P, _P, _I64, _I64, _I64, _I64, _I64, _P]),
    "im_qgemm_packed": (_INT, [_P, _P, _P, _P, _I64, _I64, _I64, _INT, _P, _I64, _P, ctypes.c_float, _INT, _P, _I64,
                               _P, _SZ, _P]),
    "im_qgemm_packed_attn_rows": (_I64, [_I64, _I64]),
    "im_qgemm_packed_attn": (_INT, [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _I64, _I64,
                                    _I64, _P, _I64, _P, _SZ, _P]),
    "im_argmax_rows": (_INT, [_P, _I64, _I64, _I64, _P, _I64, _P, _P, _SZ, _P]),
    "im_argmax_workspace_bytes": (_SZ, [_I64, _I64]),
    "im_kq_mul_mat": (_INT, [ctypes.c_int, _P, _P, _P, _I64, _I64, _I64, _P]),
    "im_kq_gemv": (_INT, [ctypes.c_int, _P, _P, _P, _I64, _I64, _I64, _P, _SZ, _P]),
    "ironmule_kg_mul_mat": (_INT, [ctypes.c_int, _P, _P, _P, _I64, _I64, _I64, _P]),
    "im_kq_workspace_bytes": (_SZ, [_I64, _I64]),
    "im_verify_greedy": (_INT, [_P, _I64, _I64, _I64, _I64, _P, _I64, _P, _P, _P, _P, _SZ, _P]),
    "im_quantize_w4g64": (_INT, [_P, _I64, _I64, _P, _P, _P, _P]),
    "im_rmsnorm": (_INT, [_P, _I64, _P, _P, _I64, _I64, ctypes.c_float, _INT, _P]),
    "im_qk_norm_rope_kv": (_INT, [_P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, ctypes.c_float,
                                  _INT, _P, _P, _P, _P]),
    "im_embed_w4g64": (_INT, [_P, _I64, _P, _P, _P, _I64, _I64, _I64, ctypes.c_float, _P, _P, _P]),
    "im_attention_paged": (_INT, [_P, _P, _P, _P, _I64, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64,
                                  _I64, _I64, _I64, ctypes.c_float, _P, _P, _SZ, _P]),
    "im_attention_workspace_bytes": (_SZ, [_I64, _I64, _I64, _I64, _I64, _I64, _I64]),
    "im_attention_tune": (_INT, [_INT]),
    "im_attention_qkv_paged": (_INT, [_P, _P, _P, _P, _P, ctypes.c_float, _INT, _P, _P, _P, _I64, _P, _P, _P, _P,
                                      _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, ctypes.c_float, _P, _P,
                                      _SZ, _P]),
    "im_spec_prepare": (_INT, [_P, _I64, _P, _P, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P]),
    "im_spec_commit": (_INT, [_P, _I64, _P, _P, _I64, _I64, _P, _P, _P, _P]),
    "im_sampling_workspace_bytes": (_SZ, [_I64]),
    "im_accept_stochastic": (_INT, [_P, _P, _I64, _I64, _I64, _I64, _P, _I64, ctypes.c_float, ctypes.c_float,
                                    ctypes.c_uint64, ctypes.c_uint64, _P, _P, _P, _P, _P, _SZ, _P]),
    "im_sample_rows": (_INT, [_P, _I64, _I64, _I64, ctypes.c_float, ctypes.c_float, ctypes.c_uint64,
                              ctypes.c_uint64, _P, _P, ctypes.c_uint32, _P, _I64, _P, _SZ, _P]),
    "im_philox4x32_10": (_INT, [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32, _P, _P]),
}


class KernelLibraryMissing(RuntimeError):
    """libimspec.so is not built or does not load. There is no fallback path."""


class KernelError(RuntimeError):
    """A libimspec entry point returned a non-zero status."""

    def __init__(self, name: str, status: int, message: str):
        super().__init__(f"{name} returned {status}: {message}")
        self.status = status


class KernelUnsupported(KernelError):
    """IM_UNSUPPORTED: the shape or mode is outside what the kernels cover; nothing was launched."""


_lib: ctypes.CDLL | None = None
_lock = threading.Lock()


def load(path: Path | None = None) -> ctypes.CDLL:
    """The loaded library (loaded once per process)."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        target = Path(path) if path is not None else LIB_PATH
        if not target.exists():
            raise KernelLibraryMissing(f"{target} is not built: run `python -m ironmule_b200.build`")
        try:
            lib = ctypes.CDLL(str(target))
        except OSError as exc:
            raise KernelLibraryMissing(f"{target} does not load: {exc}") from exc
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype, fn.argtypes = restype, argtypes
        version = lib.im_abi_version()
        if version != ABI_VERSION:
            raise KernelLibraryMissing(f"{target} implements ABI {version}, this package expects {ABI_VERSION}")
        if path is None:
            _lib = lib
        return lib


def call(name: str, *args) -> None:
    """Call an int-returning entry point and raise on a non-zero status."""
    lib = load()
    status = getattr(lib, name)(*args)
    if status != IM_OK:
        message = (lib.im_last_error() or b"").decode(errors="replace")
        cls = KernelUnsupported if status == IM_UNSUPPORTED else KernelError
        raise cls(name, status, message)
