"""Torch-facing wrappers of the libimspec kernels: device tensors in, device tensors out, the current CUDA
stream, no host synchronisation. PyTorch supplies memory and streams; the arithmetic is libimspec's.

Weights use MLX's affine 4-bit layout: `w` int32/uint32 [N, K/8] (8 codes per word, low nibble first),
`scales` and `biases` bf16 [N, K/64].

Kernels that reduce across CTAs borrow a zero-filled scratch buffer. Pass one explicitly (`ws=`, a uint8 CUDA
tensor from `workspace()`) where the call is captured in a CUDA graph or may overlap another call;
otherwise a shared per-device buffer is used.
"""
from __future__ import annotations

import ctypes
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


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    """A zero-filled scratch buffer of at least `nbytes` usable bytes (256-byte aligned inside)."""
    return torch.zeros(max(int(nbytes), 1 << 16) + 256, dtype=torch.uint8, device=device)


def _ws(buf: torch.Tensor, need: int) -> tuple[int, int]:
    ptr = buf.data_ptr()
    pad = (-ptr) % 256
    size = buf.numel() - pad
    if size < need:
        raise ValueError(f"workspace of {need} bytes needed, {size} given")
    return ptr + pad, size


class _Shared:
    """Per-(device, purpose) shared scratch for eager calls. The kernels leave counters at zero, so a buffer
    is reused as is; it grows by reallocation (never during CUDA graph capture: pass `ws=` there)."""

    buffers: dict[tuple, torch.Tensor] = {}
    lock = threading.Lock()

    @classmethod
    def get(cls, device: torch.device, need: int, purpose: str) -> torch.Tensor:
        key = (device.index, purpose)
        with cls.lock:
            buf = cls.buffers.get(key)
            if buf is None or buf.numel() - 256 < need:
                buf = workspace(need, device)
                cls.buffers[key] = buf
        return buf


def _ptr_or_none(t):
    return t.data_ptr() if t is not None else None


def _scratch(ws, device, need, purpose):
    if need == 0:
        return None, 0
    buf = ws if ws is not None else _Shared.get(device, need, purpose)
    return _ws(buf, need)


def qgemm_workspace_bytes(m: int, n: int, k: int) -> int:
    return int(_lib.load().im_qgemm_workspace_bytes(m, n, k))


def qgemm(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, *,
          epilogue: str = "store", residual: torch.Tensor | None = None, out: torch.Tensor | None = None,
          variant: str = "auto", split_k: bool = True, ws: torch.Tensor | None = None,
          rows: int | None = None) -> torch.Tensor:
    """y[M, N] = x[M, K] . dequantize(w)[N, K]^T (bf16), or a fused epilogue of it. `rows` limits M to the
    first rows of x."""
    device = x.device
    _check(x, "x", (torch.bfloat16,))
    _check(w, "w", (torch.int32, torch.uint32), device)
    _check(scales, "scales", (torch.bfloat16,), device)
    _check(biases, "biases", (torch.bfloat16,), device)
    k = x.shape[-1]
    m = x.numel() // k if rows is None else rows
    n = w.shape[0]
    if w.shape[1] * 8 != k or scales.shape != (n, k // 64) or biases.shape != (n, k // 64):
        raise ValueError(f"shape mismatch: x {tuple(x.shape)}, w {tuple(w.shape)}, scales {tuple(scales.shape)}")
    epi = _EPILOGUES[epilogue]
    n_out = n // 2 if epi in (_lib.EPI_SWIGLU, _lib.EPI_GEGLU) else n
    if out is None:
        out = torch.empty((m, n_out), dtype=torch.bfloat16, device=device)
    elif out.dtype != torch.bfloat16 or out.device != device or out.numel() < m * n_out:
        raise ValueError("out must be a bf16 tensor on x's device with room for the result")
    res_ptr = None
    if epi == _lib.EPI_RESIDUAL:
        if residual is None or residual.dtype != torch.bfloat16 or residual.numel() < m * n:
            raise ValueError("the residual epilogue needs a bf16 `residual` of the output's size")
        res_ptr = residual.data_ptr()
    need = qgemm_workspace_bytes(m, n, k) if split_k else 0
    ws_ptr, ws_bytes = _scratch(ws, device, need, "qgemm")
    _lib.call("im_qgemm_w4g64_ex", w.data_ptr(), scales.data_ptr(), biases.data_ptr(), x.data_ptr(),
              out.data_ptr(), res_ptr, m, n, k, epi, _VARIANTS[variant], ws_ptr, ws_bytes, _stream(device))
    if rows is None and out.numel() == m * n_out:
        return out.view(*x.shape[:-1], n_out)
    return out


def argmax_workspace_bytes(rows: int, v: int) -> int:
    return int(_lib.load().im_argmax_workspace_bytes(rows, v))


def argmax_rows(logits: torch.Tensor, with_conf: bool = False, *, out: torch.Tensor | None = None,
                out_stride: int = 1, conf_out: torch.Tensor | None = None, ws: torch.Tensor | None = None,
                rows: int | None = None, ld: int | None = None):
    """(argmax int32, conf float32 or None) over the last axis of bf16 logits; row r starts at element r * ld
    (default: the vocabulary size); `out` may be a strided int32 buffer (row r written at out[r * out_stride])."""
    _check(logits, "logits", (torch.bfloat16,))
    device = logits.device
    v = logits.shape[-1]
    ld = v if ld is None else ld
    rows = logits.numel() // v if rows is None else rows
    if (rows - 1) * ld + v > logits.numel():
        raise ValueError("rows * ld exceed the logits buffer")
    idx = torch.empty(rows, dtype=torch.int32, device=device) if out is None else out
    conf = conf_out if conf_out is not None else (
        torch.empty(rows, dtype=torch.float32, device=device) if with_conf else None)
    ws_ptr, ws_bytes = _scratch(ws, device, argmax_workspace_bytes(rows, v), "argmax")
    _lib.call("im_argmax_rows", logits.data_ptr(), rows, v, ld, idx.data_ptr(), out_stride,
              conf.data_ptr() if conf is not None else None, ws_ptr, ws_bytes, _stream(device))
    return idx, conf


def verify_greedy(logits: torch.Tensor, drafts: torch.Tensor, *, b: int | None = None, k: int | None = None,
                  drafts_ld: int | None = None, tokens: torch.Tensor | None = None,
                  count: torch.Tensor | None = None, picks: torch.Tensor | None = None,
                  ws: torch.Tensor | None = None):
    """Greedy acceptance for B sequences with k drafts each: logits bf16 [B*(k+1), V], drafts int32 [B, k]
    (or a strided view: pass b, k, drafts_ld). Returns (tokens int32 [B, k+1] padded with -1, count int32 [B])."""
    _check(logits, "logits", (torch.bfloat16,))
    device = logits.device
    if drafts.dtype != torch.int32 or drafts.device != device:
        raise TypeError("drafts must be int32 on the logits' device")
    if b is None:
        b, k = drafts.shape
        drafts_ld = k
    v = logits.shape[-1]
    if logits.numel() < b * (k + 1) * v:
        raise ValueError("logits must hold B*(k+1) rows")
    tokens = torch.empty((b, k + 1), dtype=torch.int32, device=device) if tokens is None else tokens
    count = torch.empty(b, dtype=torch.int32, device=device) if count is None else count
    ws_ptr, ws_bytes = _scratch(ws, device, argmax_workspace_bytes(b * (k + 1), v), "argmax")
    _lib.call("im_verify_greedy", logits.data_ptr(), b, k, v, v, drafts.data_ptr(), drafts_ld, tokens.data_ptr(),
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


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, *, gemma: bool = False,
            out: torch.Tensor | None = None, rows: int | None = None, ldx: int | None = None) -> torch.Tensor:
    """RMSNorm of `rows` rows of x (row stride `ldx` elements; default: all rows, contiguous)."""
    _check(weight, "weight", (torch.bfloat16,), x.device)
    if x.dtype != torch.bfloat16 or x.device.type != "cuda":
        raise TypeError("x must be a bf16 CUDA tensor")
    h = weight.numel()
    ldx = h if ldx is None else ldx
    rows = x.numel() // h if rows is None else rows
    out = torch.empty((rows, h), dtype=torch.bfloat16, device=x.device) if out is None else out
    _lib.call("im_rmsnorm", x.data_ptr(), ldx, weight.data_ptr(), out.data_ptr(), rows, h, float(eps),
              int(gemma), _stream(x.device))
    return out


def rmsnorm_residual(y: torch.Tensor, weight: torch.Tensor | None, h: torch.Tensor, eps: float, *, gemma: bool = False,
                     rows: int | None = None, out_sq: torch.Tensor | None = None) -> torch.Tensor:
    """h += rmsnorm(y) * w' per row, in place (Gemma-3's output norms); out_sq gets the new rows' sums of squares."""
    hsz = h.shape[-1]
    m = h.numel() // hsz if rows is None else rows
    _lib.call("im_rmsnorm_residual", y.data_ptr(), _ptr_or_none(weight), h.data_ptr(), m, hsz, float(eps), int(gemma),
              _ptr_or_none(out_sq), _stream(h.device))
    return h


def qk_norm_rope_kv(qkv: torch.Tensor, q_norm: torch.Tensor, k_norm: torch.Tensor, inv_freq: torch.Tensor,
                    row_pos: torch.Tensor, row_slot: torch.Tensor, row_seq: torch.Tensor, page_table: torch.Tensor,
                    hq: int, hkv: int, d: int, eps: float, k_cache: torch.Tensor, v_cache: torch.Tensor, *,
                    gemma: bool = False, q_out: torch.Tensor | None = None, rows: int | None = None) -> torch.Tensor:
    m = qkv.shape[0] if rows is None else rows
    q_out = torch.empty((m, hq, d), dtype=torch.bfloat16, device=qkv.device) if q_out is None else q_out
    _lib.call("im_qk_norm_rope_kv", qkv.data_ptr(), q_norm.data_ptr(), k_norm.data_ptr(), inv_freq.data_ptr(),
              row_pos.data_ptr(), row_slot.data_ptr(), row_seq.data_ptr(), page_table.data_ptr(),
              page_table.shape[-1], m, hq, hkv, d, float(eps), int(gemma), q_out.data_ptr(), k_cache.data_ptr(),
              v_cache.data_ptr(), _stream(qkv.device))
    return q_out


def embed(tokens: torch.Tensor, wq: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, *,
          mult: float = 1.0, out: torch.Tensor | None = None, rows: int | None = None,
          stride: int = 1, out_sq: torch.Tensor | None = None) -> torch.Tensor:
    """Rows tokens[0], tokens[stride], ... of the 4-bit table, dequantised (bf16 [rows, H])."""
    if tokens.dtype != torch.int32 or tokens.device.type != "cuda":
        raise TypeError("tokens must be an int32 CUDA tensor")
    v, h = wq.shape[0], wq.shape[1] * 8
    m = tokens.numel() if rows is None else rows
    out = torch.empty((m, h), dtype=torch.bfloat16, device=tokens.device) if out is None else out
    _lib.call("im_embed_w4g64", tokens.data_ptr(), stride, wq.data_ptr(), scales.data_ptr(), biases.data_ptr(), m,
              v, h, float(mult), out.data_ptr(), _ptr_or_none(out_sq), _stream(tokens.device))
    return out


def attention_workspace_bytes(b: int, rows: int, hq: int, hkv: int, d: int, max_kv_len: int, kpc: int) -> int:
    return int(_lib.load().im_attention_workspace_bytes(b, rows, hq, hkv, d, max_kv_len, kpc))


def attention_tune(waves: int) -> None:
    """Waves of resident CTAs the attention launch aims for (scheduling only; results do not change)."""
    _lib.call("im_attention_tune", int(waves))


def attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, page_table: torch.Tensor,
              seq_rows: torch.Tensor, row_slot: torch.Tensor, *, max_rows_per_seq: int, max_kv_len: int,
              scale: float, keys_per_split: int = 64, window: int = 0, tree_mask: torch.Tensor | None = None,
              tree_base: torch.Tensor | None = None, out: torch.Tensor | None = None, rows: int | None = None,
              ws: torch.Tensor | None = None, seq_slot: torch.Tensor | None = None) -> torch.Tensor:
    """Paged verification attention; q [M, Hq, D] -> out [M, Hq, D] (bf16)."""
    hq, d = q.shape[-2], q.shape[-1]
    m = q.shape[0] if rows is None else rows
    hkv = k_cache.shape[-3]
    b = seq_rows.numel() - 1
    out = torch.empty((m, hq, d), dtype=torch.bfloat16, device=q.device) if out is None else out
    need = attention_workspace_bytes(b, max_rows_per_seq, hq, hkv, d, max_kv_len, keys_per_split)
    if need == 0:
        raise ValueError("attention shape not supported")
    ws_ptr, ws_bytes = _scratch(ws, q.device, need, "attention")
    _lib.call("im_attention_paged", q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), page_table.data_ptr(),
              page_table.shape[-1], seq_rows.data_ptr(), _ptr_or_none(seq_slot), row_slot.data_ptr(),
              tree_mask.data_ptr() if tree_mask is not None else None,
              tree_base.data_ptr() if tree_base is not None else None, b, max_rows_per_seq, hq, hkv, d, max_kv_len,
              keys_per_split, window, float(scale), out.data_ptr(), ws_ptr, ws_bytes, _stream(q.device))
    return out


def attention_qkv(qkv: torch.Tensor, q_norm: torch.Tensor, k_norm: torch.Tensor, inv_freq: torch.Tensor,
                  row_pos: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, page_table: torch.Tensor,
                  seq_rows: torch.Tensor, row_slot: torch.Tensor, *, hq: int, hkv: int, d: int, eps: float,
                  max_rows_per_seq: int, max_kv_len: int, scale: float, gemma: bool = False,
                  keys_per_split: int = 64, window: int = 0, tree_mask: torch.Tensor | None = None,
                  tree_base: torch.Tensor | None = None, out: torch.Tensor | None = None, rows: int | None = None,
                  ws: torch.Tensor | None = None, seq_slot: torch.Tensor | None = None,
                  defer: bool = False) -> torch.Tensor | None:
    """Attention from the packed qkv projection rows [M, (Hq + 2 Hkv) D]: q/k RMSNorm + RoPE and the K/V cache
    write happen inside the kernel; returns out [M, Hq, D] (bf16). defer: only the split partials are written
    (into ws), for qgemm_packed_attn to merge; returns None."""
    if qkv.dtype != torch.bfloat16 or not qkv.is_contiguous():
        raise TypeError("qkv must be a contiguous bf16 tensor")
    m = qkv.shape[0] if rows is None else rows
    b = seq_rows.numel() - 1
    if defer and ws is None:
        raise ValueError("a deferred merge needs the workspace its consumer reads")
    if not defer:
        out = torch.empty((m, hq, d), dtype=torch.bfloat16, device=qkv.device) if out is None else out
    need = attention_workspace_bytes(b, max_rows_per_seq, hq, hkv, d, max_kv_len, keys_per_split)
    if need == 0:
        raise ValueError("attention shape not supported")
    ws_ptr, ws_bytes = _scratch(ws, qkv.device, need, "attention")
    _lib.call("im_attention_qkv_paged", qkv.data_ptr(), q_norm.data_ptr(), k_norm.data_ptr(), inv_freq.data_ptr(),
              row_pos.data_ptr(), float(eps), int(gemma), k_cache.data_ptr(), v_cache.data_ptr(),
              page_table.data_ptr(), page_table.shape[-1], seq_rows.data_ptr(), _ptr_or_none(seq_slot),
              row_slot.data_ptr(), _ptr_or_none(tree_mask), _ptr_or_none(tree_base), b, max_rows_per_seq, hq, hkv,
              d, max_kv_len, keys_per_split, window, float(scale), None if defer else out.data_ptr(), ws_ptr,
              ws_bytes, _stream(qkv.device))
    return None if defer else out


def spec_prepare(hist, n, target, b: int, k: int, slot_cap: int, d0_tok, d0_pos, d_pos, v_tok, v_pos) -> None:
    _lib.call("im_spec_prepare", hist.data_ptr(), hist.shape[-1], n.data_ptr(), target.data_ptr(), b, k, slot_cap,
              d0_tok.data_ptr(), d0_pos.data_ptr(), d_pos.data_ptr() if d_pos is not None else None,
              v_tok.data_ptr(), v_pos.data_ptr(), _stream(hist.device))


def spec_commit(hist, n, target, b: int, k: int, out_tokens, out_count, stats=None) -> None:
    _lib.call("im_spec_commit", hist.data_ptr(), hist.shape[-1], n.data_ptr(), target.data_ptr(), b, k,
              out_tokens.data_ptr(), out_count.data_ptr(), stats.data_ptr() if stats is not None else None,
              _stream(hist.device))


def sampling_workspace_bytes(rows: int) -> int:
    return int(_lib.load().im_sampling_workspace_bytes(rows))


def sample_rows(logits: torch.Tensor, temperature: float, top_p: float, seed: int, offset: int = 0, *,
                offset_dev: torch.Tensor | None = None, streams: torch.Tensor | None = None, draw: int = 0,
                out: torch.Tensor | None = None, out_stride: int = 1, rows: int | None = None,
                ws: torch.Tensor | None = None) -> torch.Tensor:
    """One token per row from softmax(logits / T) restricted to top-p, on the Philox stream."""
    _check(logits, "logits", (torch.bfloat16,))
    v = logits.shape[-1]
    rows = logits.numel() // v if rows is None else rows
    out = torch.empty(rows, dtype=torch.int32, device=logits.device) if out is None else out
    ws_ptr, ws_bytes = _scratch(ws, logits.device, sampling_workspace_bytes(rows), "sampling")
    _lib.call("im_sample_rows", logits.data_ptr(), rows, v, v, float(temperature), float(top_p), int(seed),
              int(offset), _ptr_or_none(offset_dev), _ptr_or_none(streams), int(draw), out.data_ptr(), out_stride,
              ws_ptr, ws_bytes, _stream(logits.device))
    return out


def accept_stochastic(target_logits: torch.Tensor, draft_logits: torch.Tensor, drafts: torch.Tensor, *, b: int,
                      k: int, drafts_ld: int, temperature: float, top_p: float, seed: int, offset: int = 0,
                      offset_dev: torch.Tensor | None = None, tokens: torch.Tensor | None = None,
                      count: torch.Tensor | None = None, ratios: torch.Tensor | None = None,
                      ws: torch.Tensor | None = None):
    """p/q rejection sampling: target_logits [B, k+1, V], draft_logits [k, B, V] -> (tokens [B, k+1], count [B])."""
    _check(target_logits, "target_logits", (torch.bfloat16,))
    _check(draft_logits, "draft_logits", (torch.bfloat16,), target_logits.device)
    device = target_logits.device
    v = target_logits.shape[-1]
    tokens = torch.empty((b, k + 1), dtype=torch.int32, device=device) if tokens is None else tokens
    count = torch.empty(b, dtype=torch.int32, device=device) if count is None else count
    ws_ptr, ws_bytes = _scratch(ws, device, sampling_workspace_bytes(b * (2 * k + 1)), "sampling")
    _lib.call("im_accept_stochastic", target_logits.data_ptr(), draft_logits.data_ptr(), b, k, v, v,
              drafts.data_ptr(), drafts_ld, float(temperature), float(top_p), int(seed), int(offset),
              _ptr_or_none(offset_dev), tokens.data_ptr(), count.data_ptr(), _ptr_or_none(ratios), ws_ptr,
              ws_bytes, _stream(device))
    return tokens, count


def topk_workspace_bytes(rows: int, v: int, k: int) -> int:
    return int(_lib.load().im_topk_workspace_bytes(rows, v, k))


def topk_rows(logits: torch.Tensor, k: int, *, rows: int | None = None, ld: int | None = None,
              out: torch.Tensor | None = None, out_stride: int | None = None,
              ws: torch.Tensor | None = None) -> torch.Tensor:
    """The k largest entries of each row (indices, largest first, ties to the lower index)."""
    _check(logits, "logits", (torch.bfloat16,))
    v = logits.shape[-1]
    ld = v if ld is None else ld
    rows = logits.numel() // v if rows is None else rows
    out_stride = k if out_stride is None else out_stride
    out = torch.empty((rows, k), dtype=torch.int32, device=logits.device) if out is None else out
    ws_ptr, ws_bytes = _scratch(ws, logits.device, topk_workspace_bytes(rows, v, k), "topk")
    _lib.call("im_topk_rows", logits.data_ptr(), rows, v, ld, k, out.data_ptr(), out_stride, ws_ptr, ws_bytes,
              _stream(logits.device))
    return out


def _branch(branch) -> ctypes.Array:
    return (ctypes.c_int32 * len(branch))(*branch)


def tree_prepare(hist, n, branch, slot_cap: int, d0_tok, d0_pos, v_tok, v_pos, v_slot, v_mask, tree_base) -> None:
    _lib.call("im_tree_prepare", hist.data_ptr(), hist.shape[-1], n.data_ptr(), n.numel(), _branch(branch),
              len(branch), slot_cap, d0_tok.data_ptr(), d0_pos.data_ptr(), v_tok.data_ptr(), v_pos.data_ptr(),
              v_slot.data_ptr(), v_mask.data_ptr(), tree_base.data_ptr(), _stream(hist.device))


def tree_accept(argmax, v_tok, b: int, branch, out_tokens, out_count, acc_node) -> None:
    _lib.call("im_tree_accept", argmax.data_ptr(), v_tok.data_ptr(), b, _branch(branch), len(branch),
              out_tokens.data_ptr(), out_count.data_ptr(), acc_node.data_ptr(), _stream(argmax.device))


def tree_compact(k_cache: torch.Tensor, v_cache: torch.Tensor, page_table, tree_base, acc_node, levels: int,
                 max_depth: int, b: int) -> None:
    """k_cache / v_cache [layers, pages, Hkv, 16, D]."""
    layers, _, hkv, _, d = k_cache.shape
    _lib.call("im_tree_compact", k_cache.data_ptr(), v_cache.data_ptr(), layers, k_cache.stride(0),
              page_table.data_ptr(), page_table.shape[-1], tree_base.data_ptr(), acc_node.data_ptr(), levels,
              max_depth, b, hkv, d, _stream(k_cache.device))


def philox(seed: int, offset: int, stream_id: int, n: int, device) -> torch.Tensor:
    out = torch.empty((n, 4), dtype=torch.int32, device=device)
    _lib.call("im_philox4x32_10", int(seed), int(offset), int(stream_id), int(n), out.data_ptr(), _stream(device))
    return out


# ---- packed weights (the engine's resident format) ------------------------------------------------------
class Packed:
    """A 4-bit projection repacked into MMA-fragment order (im_qgemm_pack_w4g64): n rows, k inputs."""

    def __init__(self, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor):
        _check(w, "w", (torch.int32, torch.uint32))
        self.n, self.k = int(w.shape[0]), int(w.shape[1]) * 8
        nbytes = int(_lib.load().im_qgemm_packed_bytes(self.n, self.k))
        self.data = torch.empty(nbytes, dtype=torch.uint8, device=w.device)
        _lib.call("im_qgemm_pack_w4g64", w.data_ptr(), scales.data_ptr(), biases.data_ptr(), self.n, self.k,
                  self.data.data_ptr(), _stream(w.device))

    @property
    def tiles(self) -> int:
        return (self.n + 31) // 32


def set_launch_overlap(on: bool) -> bool:
    """Programmatic dependent launch of the decode-path kernels on (default) or off; returns the previous
    setting. Results are bit-identical either way."""
    return bool(_lib.load().im_set_launch_overlap(int(bool(on))))


def qgemm_packed_workspace_bytes(m: int, n: int, k: int) -> int:
    return int(_lib.load().im_qgemm_packed_workspace_bytes(m, n, k))


def qgemm_packed_status(ws: torch.Tensor) -> int:
    """The error word of a workspace last used by a call of more than 32 rows (0: every wait completed)."""
    ptr, _ = _ws(ws, 1 << 16)
    return int(_lib.load().im_qgemm_packed_status(ptr))


def qgemm_packed_path(path: int) -> None:
    """0: automatic (default); 1: warp MMA always; 2: tcgen05 tensor cores always. Every choice gives the same
    bits."""
    _lib.call("im_qgemm_packed_path", int(path))


def qgemm_packed_cluster(on: bool) -> None:
    """Split-K partials of the warp-MMA kernel summed inside a thread-block cluster (True, default) or through
    the workspace and a global counter (False). Both give the same bits."""
    _lib.call("im_qgemm_packed_cluster", int(bool(on)))


def qgemm_packed_tune(split_override: int = 0, target_ctas: int = 592, max_split: int = 16) -> None:
    """The K-split policy (process-wide; changes workspace sizes)."""
    _lib.call("im_qgemm_packed_tune", split_override, target_ctas, max_split)


def qgemm_packed(x: torch.Tensor, p: Packed, *, epilogue: str = "store", residual: torch.Tensor | None = None,
                 out: torch.Tensor | None = None, rows: int | None = None, norm_sq: torch.Tensor | None = None,
                 norm_parts: int = 0, norm_weight: torch.Tensor | None = None, eps: float = 1e-6,
                 gemma_norm: bool = False, out_sq: torch.Tensor | None = None, sq_ld: int = 0,
                 ws: torch.Tensor | None = None) -> torch.Tensor:
    """y = x . W^T over packed weights, with an optional fused RMSNorm prologue (norm_sq/norm_weight) and
    per-tile sums of squares of the output (out_sq)."""
    device = x.device
    if x.dtype != torch.bfloat16 or device.type != "cuda" or not x.is_contiguous():
        raise TypeError("x must be a contiguous bf16 CUDA tensor")
    k = x.shape[-1]
    if k != p.k:
        raise ValueError(f"x has K={k}, the weights {p.k}")
    m = x.numel() // k if rows is None else rows
    epi = _EPILOGUES[epilogue]
    n_out = p.n // 2 if epi in (_lib.EPI_SWIGLU, _lib.EPI_GEGLU) else p.n
    out = torch.empty((m, n_out), dtype=torch.bfloat16, device=device) if out is None else out
    ws_ptr, ws_bytes = _scratch(ws, device, qgemm_packed_workspace_bytes(m, p.n, p.k), "qgemm_packed")
    _lib.call("im_qgemm_packed", p.data.data_ptr(), x.data_ptr(), out.data_ptr(), _ptr_or_none(residual), m, p.n, p.k,
              epi, _ptr_or_none(norm_sq), norm_parts, _ptr_or_none(norm_weight), float(eps), int(gemma_norm),
              _ptr_or_none(out_sq), sq_ld, ws_ptr, ws_bytes, _stream(device))
    return out


def qgemm_packed_attn_rows(n: int, k: int) -> int:
    """The most rows qgemm_packed_attn takes for an [n, k] projection (0: none)."""
    return int(_lib.load().im_qgemm_packed_attn_rows(n, k))


def qgemm_packed_attn(attn_ws: torch.Tensor, p: Packed, seq_rows: torch.Tensor, row_slot: torch.Tensor, *,
                      residual: torch.Tensor, out: torch.Tensor, rows: int, max_rows_per_seq: int, hq: int, hkv: int,
                      d: int, max_kv_len: int, keys_per_split: int, out_sq: torch.Tensor | None = None,
                      sq_ld: int = 0, ws: torch.Tensor | None = None) -> torch.Tensor:
    """The o-projection with a residual epilogue whose input is the attention output merged, in its prologue,
    from the split partials that attention_qkv(..., defer=True) left in attn_ws (the same bits as merging them
    in the attention and projecting its output). Takes at most qgemm_packed_attn_rows(p.n, p.k) rows."""
    device = residual.device
    b = seq_rows.numel() - 1
    ws_ptr, ws_bytes = _scratch(ws, device, qgemm_packed_workspace_bytes(rows, p.n, p.k), "qgemm_packed")
    _lib.call("im_qgemm_packed_attn", p.data.data_ptr(), attn_ws.data_ptr(), seq_rows.data_ptr(), row_slot.data_ptr(),
              b, max_rows_per_seq, hq, hkv, d, max_kv_len, keys_per_split, out.data_ptr(), residual.data_ptr(), rows,
              p.n, p.k, _ptr_or_none(out_sq), sq_ld, ws_ptr, ws_bytes, _stream(device))
    return out


# ---- GGUF k-quants (the ggml path) ----------------------------------------------------------------------------
Q4_K, Q6_K = 12, 14
KQ_BLOCK_BYTES = {Q4_K: 144, Q6_K: 210}


def kq_workspace_bytes(k: int, b: int) -> int:
    return int(_lib.load().im_kq_workspace_bytes(k, b))


def _kq_args(kind: int, w: torch.Tensor, x: torch.Tensor, n: int, out: torch.Tensor | None):
    if kind not in KQ_BLOCK_BYTES:
        raise ValueError(f"weight type {kind}: 12 (Q4_K) or 14 (Q6_K)")
    _check(w, "w", (torch.uint8,))
    _check(x, "x", (torch.float32,), w.device)
    if x.dim() != 2:
        raise ValueError("x must be [B, K]")
    b, k = x.shape
    if k % 256 or w.numel() != n * (k // 256) * KQ_BLOCK_BYTES[kind]:
        raise ValueError(f"w holds {w.numel()} bytes, expected {n} rows of {k // 256} blocks")
    y = torch.empty((b, n), dtype=torch.float32, device=w.device) if out is None else out
    _check(y, "out", (torch.float32,), w.device)
    if tuple(y.shape) != (b, n):
        raise ValueError(f"out must be [{b}, {n}]")
    return b, k, y


def kq_gemv(kind: int, w: torch.Tensor, x: torch.Tensor, n: int, *, out: torch.Tensor | None = None,
            ws: torch.Tensor | None = None) -> torch.Tensor:
    """y [B, N] float32 = x [B, K] float32 . W^T, W = N rows of GGUF Q4_K / Q6_K blocks as raw bytes (uint8)."""
    b, k, y = _kq_args(kind, w, x, n, out)
    ws_ptr, ws_bytes = _scratch(ws, w.device, kq_workspace_bytes(k, b), "kq")
    _lib.call("im_kq_gemv", kind, w.data_ptr(), x.data_ptr(), y.data_ptr(), n, k, b, ws_ptr, ws_bytes,
              _stream(w.device))
    return y


def kq_mul_mat(kind: int, w: torch.Tensor, x: torch.Tensor, n: int, *,
               out: torch.Tensor | None = None) -> tuple[int, torch.Tensor]:
    """The llama.cpp hook's call (`ironmule_kg_mul_mat`): (0, y) when y was computed, else (the library's refusal
    code, y unwritten) and the caller runs its own kernel."""
    b, k, y = _kq_args(kind, w, x, n, out)
    rc = int(_lib.load().im_kq_mul_mat(kind, w.data_ptr(), x.data_ptr(), y.data_ptr(), n, k, b,
                                       _stream(w.device)))
    return rc, y
