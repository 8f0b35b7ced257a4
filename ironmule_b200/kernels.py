"""Torch-facing wrappers of the libimspec kernels: device tensors in, device tensors out, the current CUDA
stream, no host synchronisation. PyTorch supplies memory and streams; the arithmetic is libimspec's.

Weights use MLX's affine 4-bit layout: `w` int32/uint32 [N, K/8] (8 codes per word, low nibble first),
`scales` and `biases` bf16 [N, K/64].
"""
from __future__ import annotations

import threading

import torch

from . import _lib

_EPILOGUES = {"store": _lib.EPI_STORE, "residual": _lib.EPI_RESIDUAL, "swiglu": _lib.EPI_SWIGLU,
              "geglu": _lib.EPI_GEGLU}
_VARIANTS = {"auto": _lib.QGEMM_AUTO, "mma": _lib.QGEMM_MMA, "fma": _lib.QGEMM_FMA}


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _check(t: torch.Tensor, name: str, dtypes: tuple, device: torch.device | None = None) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor (there is no CPU path), got {t.device}")
    if device is not None and t.device != device:
        raise ValueError(f"{name} is on {t.device}, expected {device}")
    if t.dtype not in dtypes:
        raise TypeError(f"{name} has dtype {t.dtype}, expected one of {dtypes}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


class Workspace:
    """Zero-filled scratch buffers the kernels borrow (split-K partials, reduction counters). One buffer per
    (device, stream, purpose); the kernels leave their counters at zero, so a buffer is reused as is. Grow
    it before capturing a CUDA graph: allocation is not allowed during capture."""

    _buffers: dict[tuple, torch.Tensor] = {}
    _lock = threading.Lock()

    @classmethod
    def get(cls, device: torch.device, nbytes: int, purpose: str) -> torch.Tensor:
        key = (device.index, torch.cuda.current_stream(device).cuda_stream, purpose)
        with cls._lock:
            buf = cls._buffers.get(key)
            if buf is None or buf.numel() < nbytes:
                size = max(nbytes, 1 << 16)
                buf = torch.zeros(size + 256, dtype=torch.uint8, device=device)
                cls._buffers[key] = buf
        return buf

    @staticmethod
    def aligned_ptr(buf: torch.Tensor) -> tuple[int, int]:
        ptr = buf.data_ptr()
        pad = (-ptr) % 256
        return ptr + pad, buf.numel() - pad


def qgemm(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, *,
          epilogue: str = "store", residual: torch.Tensor | None = None, out: torch.Tensor | None = None,
          variant: str = "auto", split_k: bool = True) -> torch.Tensor:
    """y[M, N] = x[M, K] . dequantize(w)[N, K]^T (bf16), or a fused epilogue of it."""
    device = x.device
    _check(x, "x", (torch.bfloat16,))
    _check(w, "w", (torch.int32, torch.uint32), device)
    _check(scales, "scales", (torch.bfloat16,), device)
    _check(biases, "biases", (torch.bfloat16,), device)
    x2 = x.reshape(-1, x.shape[-1])
    m, k = x2.shape
    n = w.shape[0]
    if w.shape[1] * 8 != k or scales.shape != (n, k // 64) or biases.shape != (n, k // 64):
        raise ValueError(f"shape mismatch: x {tuple(x.shape)}, w {tuple(w.shape)}, scales {tuple(scales.shape)}")
    epi = _EPILOGUES[epilogue]
    n_out = n // 2 if epi in (_lib.EPI_SWIGLU, _lib.EPI_GEGLU) else n
    if out is None:
        out = torch.empty((m, n_out), dtype=torch.bfloat16, device=device)
    else:
        _check(out, "out", (torch.bfloat16,), device)
        if out.numel() != m * n_out:
            raise ValueError("out has the wrong size")
    res_ptr = None
    if epi == _lib.EPI_RESIDUAL:
        if residual is None:
            raise ValueError("the residual epilogue needs `residual`")
        _check(residual, "residual", (torch.bfloat16,), device)
        if residual.numel() != m * n:
            raise ValueError("residual has the wrong size")
        res_ptr = residual.data_ptr()
    ws_ptr, ws_bytes = None, 0
    if split_k:
        need = _lib.load().im_qgemm_workspace_bytes(m, n, k)
        if need:
            ws_ptr, ws_bytes = Workspace.aligned_ptr(Workspace.get(device, need + 256, "qgemm"))
    _lib.call("im_qgemm_w4g64_ex", w.data_ptr(), scales.data_ptr(), biases.data_ptr(), x2.data_ptr(),
              out.data_ptr(), res_ptr, m, n, k, epi, _VARIANTS[variant], ws_ptr, ws_bytes, _stream(device))
    return out.view(*x.shape[:-1], n_out)


def argmax_rows(logits: torch.Tensor, with_conf: bool = False):
    """(argmax int32 [rows], conf float32 [rows] or None) over the last axis of bf16 logits."""
    _check(logits, "logits", (torch.bfloat16,))
    device = logits.device
    rows, v = logits.reshape(-1, logits.shape[-1]).shape
    idx = torch.empty(rows, dtype=torch.int32, device=device)
    conf = torch.empty(rows, dtype=torch.float32, device=device) if with_conf else None
    need = _lib.load().im_argmax_workspace_bytes(rows, v)
    ws_ptr, ws_bytes = Workspace.aligned_ptr(Workspace.get(device, need + 256, "argmax"))
    _lib.call("im_argmax_rows", logits.data_ptr(), rows, v, v, idx.data_ptr(),
              conf.data_ptr() if conf is not None else None, ws_ptr, ws_bytes, _stream(device))
    return idx, conf


def verify_greedy(logits: torch.Tensor, drafts: torch.Tensor, *, tokens: torch.Tensor | None = None,
                  count: torch.Tensor | None = None, picks: torch.Tensor | None = None):
    """Greedy acceptance for B sequences with k drafts: logits bf16 [B*(k+1), V], drafts int32 [B, k].
    Returns (tokens int32 [B, k+1] padded with -1, count int32 [B])."""
    _check(logits, "logits", (torch.bfloat16,))
    device = logits.device
    _check(drafts, "drafts", (torch.int32,), device)
    b, k = drafts.shape
    v = logits.shape[-1]
    if logits.numel() != b * (k + 1) * v:
        raise ValueError("logits must hold B*(k+1) rows")
    tokens = torch.empty((b, k + 1), dtype=torch.int32, device=device) if tokens is None else tokens
    count = torch.empty(b, dtype=torch.int32, device=device) if count is None else count
    need = _lib.load().im_argmax_workspace_bytes(b * (k + 1), v)
    ws_ptr, ws_bytes = Workspace.aligned_ptr(Workspace.get(device, need + 256, "argmax"))
    _lib.call("im_verify_greedy", logits.data_ptr(), b, k, v, v, drafts.data_ptr(), tokens.data_ptr(),
              count.data_ptr(), picks.data_ptr() if picks is not None else None, ws_ptr, ws_bytes,
              _stream(device))
    return tokens, count


def quantize(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """MLX-affine 4-bit, group-64 quantisation of bf16 w [N, K] on the device -> (wq int32 [N, K/8],
    scales bf16 [N, K/64], biases bf16 [N, K/64])."""
    _check(w, "w", (torch.bfloat16,))
    n, k = w.shape
    if k % 64:
        raise ValueError("K must be a multiple of 64")
    wq = torch.empty((n, k // 8), dtype=torch.int32, device=w.device)
    scales = torch.empty((n, k // 64), dtype=torch.bfloat16, device=w.device)
    biases = torch.empty((n, k // 64), dtype=torch.bfloat16, device=w.device)
    _lib.call("im_quantize_w4g64", w.data_ptr(), n, k, wq.data_ptr(), scales.data_ptr(), biases.data_ptr(),
              _stream(w.device))
    return wq, scales, biases
