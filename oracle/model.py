"""TEST INFRASTRUCTURE ONLY: CPU restatement of the decode/verify forward the engine runs, for parity tests.

Layer math (numpy, float32 with bf16 rounding at every op boundary, float64 attention softmax):
  rmsnorm       out = bf16((x * 1/sqrt(mean(x^2) + eps)) * w')       w' = w (Qwen3) or 1 + w (Gemma-3)
  q/k norm      the same over head_dim with q_norm / k_norm
  rope          non-interleaved pairs (i, i + D/2), angle = float32(pos) * inv_freq[i], inv_freq = theta^(-2i/D)
  attention     softmax((q . k) * scale) . v over the row's visible slots (causal, window, tree)
  swiglu        bf16(bf16(a * bf16(sigmoid(a))) * u), a = bf16(gate), u = bf16(up)
  residual      bf16(h + bf16(y))
  embedding     bf16(scale * q + bias) of the token's row (x bf16(sqrt(H)) for Gemma-3)
  Gemma-3       RMSNorm of the attention output and of the MLP output ((1 + w) weights) before each residual add
Projections go through `oracle.qmv.qmv`, the pinned restatement of the reference's qmv arithmetic
(IronMule ironmule/qmv_k3840.py:62-244). The decode-layer order follows mlx_lm's Qwen3 as the reference's
runtime drives it (ironmule/runtime.py:505-545) and the Gemma-3 decode step of
ironmule/paired_research.py:177-215; the stacked-plan conventions (slots, per-row lengths) follow
ironmule/dense_plan.py:337-363.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

from . import bf16, qmv, quant

R = bf16.round_f32


def rmsnorm(x_bits: np.ndarray, w_bits: np.ndarray, eps: float, gemma: bool = False) -> np.ndarray:
    x = bf16.to_f32(x_bits)
    ms = np.sum(x * x, axis=-1, dtype=np.float32, keepdims=True) / np.float32(x.shape[-1])
    inv = np.float32(1.0) / np.sqrt(ms + np.float32(eps))
    w = bf16.to_f32(w_bits)
    w = (np.float32(1.0) + w) if gemma else w
    return bf16.from_f32((x * inv) * w)


def rope(x_f32: np.ndarray, pos: np.ndarray, inv_freq: np.ndarray) -> np.ndarray:
    """x [M, H, D] float32 (already bf16-valued), pos [M] -> bf16 bits."""
    d = x_f32.shape[-1]
    half = d // 2
    ang = pos.astype(np.float32)[:, None] * inv_freq[None, :]             # float32 [M, D/2]
    c = np.cos(ang.astype(np.float64)).astype(np.float32)[:, None, :]
    s = np.sin(ang.astype(np.float64)).astype(np.float32)[:, None, :]
    x1, x2 = x_f32[..., :half], x_f32[..., half:]
    return bf16.from_f32(np.concatenate([x1 * c - x2 * s, x1 * s + x2 * c], axis=-1))


def silu_mul(gate_bits: np.ndarray, up_bits: np.ndarray) -> np.ndarray:
    a, u = bf16.to_f32(gate_bits), bf16.to_f32(up_bits)
    sig = R((1.0 / (1.0 + np.exp(-a.astype(np.float64)))).astype(np.float32))
    return bf16.from_f32(R(a * sig) * u)


def gelu_mul(gate_bits: np.ndarray, up_bits: np.ndarray) -> np.ndarray:
    a, u = bf16.to_f32(gate_bits), bf16.to_f32(up_bits)
    inner = np.float32(0.7978845608028654) * (a + np.float32(0.044715) * a * a * a)
    ge = R((0.5 * a * (1.0 + np.tanh(inner.astype(np.float64)))).astype(np.float32))
    return bf16.from_f32(ge * u)


def residual(h_bits: np.ndarray, y_bits: np.ndarray) -> np.ndarray:
    return bf16.from_f32(bf16.to_f32(h_bits) + bf16.to_f32(y_bits))


def attention(q_bits, k_bits, v_bits, row_slot, scale, window=0, tree_mask=None, tree_base=0):
    """q [M, Hq, D] bits; k, v [S, Hkv, D] bits of ONE sequence (slot-indexed); row_slot [M]. -> [M, Hq, D] bits.
    Row r sees slot s iff s <= row_slot[r], s > row_slot[r] - window (window > 0), and for s >= tree_base
    (tree mode) bit (s - tree_base) of tree_mask[r]."""
    q = bf16.to_f32(q_bits).astype(np.float64)
    k = bf16.to_f32(k_bits).astype(np.float64)
    v = bf16.to_f32(v_bits).astype(np.float64)
    m, hq, d = q.shape
    hkv = k.shape[1]
    g = hq // hkv
    out = np.zeros((m, hq, d), dtype=np.float32)
    slots = np.arange(k.shape[0])
    for r in range(m):
        vis = slots <= row_slot[r]
        if window > 0:
            vis &= slots > row_slot[r] - window
        if tree_mask is not None:
            node = slots - tree_base
            bit = np.array([(int(tree_mask[r]) >> int(n)) & 1 if 0 <= n < 64 else (1 if n < 0 else 0)
                            for n in node], dtype=bool)
            vis &= bit
        idx = np.nonzero(vis)[0]
        if idx.size == 0:
            continue
        for h in range(hq):
            kh = h // g
            sc = (k[idx, kh, :] @ q[r, h, :]) * scale
            p = np.exp(sc - sc.max())
            out[r, h] = (p @ v[idx, kh, :]) / p.sum()
    return bf16.from_f32(out)


@dataclass
class HostLayer:
    qkv: tuple
    o: tuple
    gate_up: tuple
    down: tuple
    in_norm: np.ndarray
    post_norm: np.ndarray
    q_norm: np.ndarray
    k_norm: np.ndarray
    post_attn_norm: np.ndarray | None = None   # Gemma-3 only
    post_ff_norm: np.ndarray | None = None


class OracleModel:
    """The engine's forward on the CPU, over weights copied from a device model (`from_device`)."""

    def __init__(self, cfg, embed, layers, final_norm, inv_freq, inv_freq_local, fast: bool = False):
        self.cfg = cfg
        # fast=True projects with the dequantise-and-dot CPU routine (the timed CPU baseline) instead of the
        # order-exact restatement of the reference's qmv arithmetic (the parity checker)
        self.proj = qmv.qmm_fast if fast else qmv.qmv
        self.embed, self.layers, self.final_norm = embed, layers, final_norm
        self.inv_freq, self.inv_freq_local = inv_freq, inv_freq_local
        self.k = [None] * cfg.layers  # per layer [slots, Hkv, D] bits of sequence 0
        self.v = [None] * cfg.layers

    @classmethod
    def from_device(cls, model, fast: bool = False) -> "OracleModel":
        import torch

        def host_lin(lin):
            return (lin.w.cpu().numpy().view(np.uint32), lin.s.view(torch.int16).cpu().numpy().view(np.uint16),
                    lin.b.view(torch.int16).cpu().numpy().view(np.uint16))

        def host_vec(t):
            return t.view(torch.int16).cpu().numpy().view(np.uint16)

        layers = [HostLayer(host_lin(l.qkv), host_lin(l.o), host_lin(l.gate_up), host_lin(l.down), host_vec(l.in_norm),
                            host_vec(l.post_norm), host_vec(l.q_norm), host_vec(l.k_norm),
                            host_vec(l.post_attn_norm) if l.post_attn_norm is not None else None,
                            host_vec(l.post_ff_norm) if l.post_ff_norm is not None else None) for l in model.layers]
        return cls(model.cfg, host_lin(model.embed), layers, host_vec(model.final_norm),
                   model.inv_freq.cpu().numpy(), model.inv_freq_local.cpu().numpy(), fast=fast)

    def reset(self, slots: int) -> None:
        c = self.cfg
        for li in range(c.layers):
            self.k[li] = np.zeros((slots, c.kv_heads, c.head_dim), dtype=np.uint16)
            self.v[li] = np.zeros((slots, c.kv_heads, c.head_dim), dtype=np.uint16)

    def embed_rows(self, tokens: list[int]) -> np.ndarray:
        """The rows' hidden states after the embedding gather (bf16 bits [M, H])."""
        c = self.cfg
        wq, s, b = self.embed
        h = quant.dequantize_bf16(wq[tokens], s[tokens], b[tokens])
        if c.family == "gemma3":
            h = bf16.from_f32(bf16.to_f32(h) * R(np.float32(math.sqrt(c.hidden))))
        return h

    def layer_forward(self, li: int, h: np.ndarray, slots, positions=None, tree_mask=None,
                      tree_base: int = 0) -> np.ndarray:
        """Decoder layer `li` over hidden rows h (bits [M, H]) of sequence 0: writes the rows' K/V at `slots` of
        this layer's cache and returns the layer's output rows. Positions (RoPE) default to the slots; a tree
        verify passes both, with each row's ancestor bits over the slots from tree_base on."""
        c = self.cfg
        gemma = c.family == "gemma3"
        layer = self.layers[li]
        m = h.shape[0]
        slots = np.asarray(slots)
        pos = slots if positions is None else np.asarray(positions)
        glob = c.is_global(li)
        xn = rmsnorm(h, layer.in_norm, c.eps, gemma)
        qkv = self.proj(*layer.qkv, xn).reshape(m, c.heads + 2 * c.kv_heads, c.head_dim)
        q, k, v = qkv[:, :c.heads], qkv[:, c.heads:c.heads + c.kv_heads], qkv[:, c.heads + c.kv_heads:]
        inv_freq = self.inv_freq if glob else self.inv_freq_local
        qn = bf16.to_f32(rmsnorm(q, layer.q_norm, c.eps, gemma))
        kn = bf16.to_f32(rmsnorm(k, layer.k_norm, c.eps, gemma))
        q_rot, k_rot = rope(qn, pos, inv_freq), rope(kn, pos, inv_freq)
        self.k[li][slots] = k_rot
        self.v[li][slots] = v
        att = attention(q_rot, self.k[li], self.v[li], slots, c.scale, 0 if glob else c.sliding_window,
                        tree_mask=tree_mask, tree_base=tree_base)
        y = self.proj(*layer.o, att.reshape(m, -1))
        if gemma:  # Gemma-3: post_attention_layernorm on the attention output
            y = rmsnorm(y, layer.post_attn_norm, c.eps, gemma)
        h = residual(h, y)
        xn = rmsnorm(h, layer.post_norm, c.eps, gemma)
        gu = self.proj(*layer.gate_up, xn).reshape(m, -1, 2, 16)
        gate, up = gu[:, :, 0, :].reshape(m, -1), gu[:, :, 1, :].reshape(m, -1)
        act = gelu_mul(gate, up) if gemma else silu_mul(gate, up)
        y = self.proj(*layer.down, act)
        if gemma:  # Gemma-3: post_feedforward_layernorm on the MLP output
            y = rmsnorm(y, layer.post_ff_norm, c.eps, gemma)
        return residual(h, y)

    def layer_steps(self, li: int, dev: dict, slots, positions=None, tree_mask=None, tree_base: int = 0) -> dict:
        """Each op of layer `li` restated from the DEVICE's input to that op (bits in `dev`: "h_in", "qkv", "attn",
        "h_mid", "act", and "h_out" = the next layer's input), so every op is checked with identical inputs:
          "qkv"    projection of the input RMSNorm of h_in
          "attn"   q/k RMSNorm + RoPE of the device's qkv, K/V written at `slots`, attention over the cache
          "h_mid"  h_in + o(attn)                     (Gemma-3: + RMSNorm of o(attn))
          "act"    SwiGLU / GeGLU of gate_up(RMSNorm(h_mid))
          "h_out"  h_mid + down(act)                  (Gemma-3: + RMSNorm of down(act))"""
        c = self.cfg
        gemma = c.family == "gemma3"
        layer = self.layers[li]
        m = dev["h_in"].shape[0]
        slots = np.asarray(slots)
        pos = slots if positions is None else np.asarray(positions)
        glob = c.is_global(li)
        out = {"qkv": self.proj(*layer.qkv, rmsnorm(dev["h_in"], layer.in_norm, c.eps, gemma))}
        qkv = dev["qkv"].reshape(m, c.heads + 2 * c.kv_heads, c.head_dim)
        q, k, v = qkv[:, :c.heads], qkv[:, c.heads:c.heads + c.kv_heads], qkv[:, c.heads + c.kv_heads:]
        inv_freq = self.inv_freq if glob else self.inv_freq_local
        q_rot = rope(bf16.to_f32(rmsnorm(q, layer.q_norm, c.eps, gemma)), pos, inv_freq)
        self.k[li][slots] = rope(bf16.to_f32(rmsnorm(k, layer.k_norm, c.eps, gemma)), pos, inv_freq)
        self.v[li][slots] = v
        out["attn"] = attention(q_rot, self.k[li], self.v[li], slots, c.scale, 0 if glob else c.sliding_window,
                                tree_mask=tree_mask, tree_base=tree_base).reshape(m, -1)
        y = self.proj(*layer.o, dev["attn"])
        if gemma:
            y = rmsnorm(y, layer.post_attn_norm, c.eps, gemma)
        out["h_mid"] = residual(dev["h_in"], y)
        gu = self.proj(*layer.gate_up, rmsnorm(dev["h_mid"], layer.post_norm, c.eps, gemma)).reshape(m, -1, 2, 16)
        gate, up = gu[:, :, 0, :].reshape(m, -1), gu[:, :, 1, :].reshape(m, -1)
        out["act"] = gelu_mul(gate, up) if gemma else silu_mul(gate, up)
        y = self.proj(*layer.down, dev["act"])
        if gemma:
            y = rmsnorm(y, layer.post_ff_norm, c.eps, gemma)
        out["h_out"] = residual(dev["h_mid"], y)
        return out

    def head(self, h: np.ndarray) -> np.ndarray:
        """Final RMSNorm and the tied head: logits bits [M, V]."""
        hn = rmsnorm(h, self.final_norm, self.cfg.eps, self.cfg.family == "gemma3")
        return self.proj(*self.embed, hn)

    def forward(self, tokens: list[int], slots: list[int], logits: bool = True) -> np.ndarray | None:
        """Rows of sequence 0 at the given slots (written to the cache); returns logits bits [M, V]."""
        h = self.embed_rows(tokens)
        for li in range(self.cfg.layers):
            h = self.layer_forward(li, h, slots)
        return self.head(h) if logits else None
