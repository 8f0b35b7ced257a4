"""MLX 4-bit checkpoints for the device engine.

The reference loads its models with `mlx_lm.load` (ironmule/tune.py:344-355) from a local snapshot whose
`config.json` declares `quantization.{bits, group_size}` (checked at ironmule/model_identity.py:201-212; the
architecture is `model_type`, :143-152). Such a snapshot (as `mlx_lm.convert --q-bits 4 --q-group-size 64`
writes it) holds every projection in MLX's affine 4-bit layout -- `<name>.weight` uint32 [N, K/8] (8 codes per
word, low nibble first), `<name>.scales` and `<name>.biases` bf16 [N, K/64] -- and the norms as bf16 vectors.
`load_mlx_4bit` reads it into a `QuantModel` without touching the quantised values: q/k/v rows are stacked into
the engine's qkv projection, gate/up rows interleaved in 16-row blocks, and each projection is repacked once into
the resident MMA-fragment format. `save_mlx_4bit` writes a `QuantModel` back in the same layout (tests round-trip
through it; it also turns the random-init benchmark models into real-format snapshots).

Architectures: Qwen3 (`model_type` "qwen3": q/k RMSNorm, SwiGLU, tied or separate head) and Gemma-3 text
(`gemma3_text`, or `gemma3` with its text model under `text_config` / `language_model.`: (1 + w) norms, post
norms, GeGLU, sliding-window layers, scaled embeddings, linear RoPE scaling of the global layers).
"""
from __future__ import annotations

import json
from pathlib import Path

import torch

from . import kernels
from .engine import Layer, Linear4, ModelConfig, QuantModel, interleave_gate_up, tp_shard


class CheckpointError(ValueError):
    """The snapshot is not an MLX 4-bit (group 64) Qwen3 / Gemma-3 checkpoint this engine can run."""


# ---- config.json --------------------------------------------------------------------------------------------
def quantisation(config: dict) -> dict:
    """The snapshot's quantisation record, with the reference's checks (positive integer bits and group size),
    restricted to what the engine runs: 4 bits, groups of 64."""
    value = config.get("quantization") or config.get("quantization_config")
    if not isinstance(value, dict):
        raise CheckpointError("config.json declares no quantization (a dense checkpoint: quantise it to 4 bits first)")
    for name in ("bits", "group_size"):
        field = value.get(name)
        if isinstance(field, bool) or not isinstance(field, int) or field <= 0:
            raise CheckpointError(f"quantization.{name} must be a positive integer")
    if value["bits"] != 4 or value["group_size"] != 64:
        raise CheckpointError(f"only 4-bit groups of 64 run here, not {value['bits']}-bit groups of "
                              f"{value['group_size']}")
    return value


def model_config(config: dict, name: str = "checkpoint") -> ModelConfig:
    """A `ModelConfig` from an MLX / Hugging Face `config.json` (text model)."""
    text = dict(config.get("text_config") or {})
    merged = {**config, **text}
    model_type = str(merged.get("model_type") or "").strip()
    if not model_type:
        raise CheckpointError("config.json names no model_type")
    family = "gemma3" if model_type.startswith("gemma3") else model_type
    if family not in ("qwen3", "gemma3"):
        raise CheckpointError(f"model_type {model_type!r}: this engine runs qwen3 and gemma3")
    try:
        hidden = int(merged["hidden_size"])
        heads = int(merged["num_attention_heads"])
        kw = dict(hidden=hidden, layers=int(merged["num_hidden_layers"]), heads=heads,
                  kv_heads=int(merged.get("num_key_value_heads", heads)),
                  head_dim=int(merged.get("head_dim") or hidden // heads),
                  inter=int(merged["intermediate_size"]), vocab=int(merged["vocab_size"]))
    except (KeyError, TypeError, ValueError) as exc:
        raise CheckpointError(f"config.json lacks a model dimension: {exc}") from exc
    extra = dict(rope_theta=float(merged.get("rope_theta", 1_000_000.0)), eps=float(merged.get("rms_norm_eps", 1e-6)),
                 family=family)
    scaling = merged.get("rope_scaling")
    if scaling:
        kind = scaling.get("rope_type", scaling.get("type"))
        if kind != "linear":
            raise CheckpointError(f"rope_scaling {kind!r} is not supported (linear only)")
        extra["rope_scale"] = float(scaling["factor"])
    if family == "gemma3":
        extra.update(sliding_window=int(merged.get("sliding_window", 0) or 0),
                     global_every=int(merged.get("sliding_window_pattern", 6) or 0),
                     rope_local_theta=float(merged.get("rope_local_base_freq", 10_000.0)),
                     query_scale=float(merged.get("query_pre_attn_scalar", kw["head_dim"])) ** -0.5)
    if kw["head_dim"] not in (128, 256):
        raise CheckpointError(f"head_dim {kw['head_dim']}: the attention kernels take 128 or 256")
    return ModelConfig(name, **kw, **extra)


# ---- tensors ------------------------------------------------------------------------------------------------
def read_tensors(root: Path) -> dict[str, torch.Tensor]:
    """Every tensor of the snapshot's safetensors files (CPU), under names with any multimodal prefix removed."""
    from safetensors.torch import load_file

    files = sorted(root.glob("*.safetensors"))
    if not files:
        raise CheckpointError(f"no safetensors files in {root}")
    out: dict[str, torch.Tensor] = {}
    for path in files:
        for name, t in load_file(str(path)).items():
            if name.startswith("language_model."):
                name = name[len("language_model."):]
            out[name] = t
    return out


def _q(weights: dict, name: str) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    try:
        w, s, b = weights[f"{name}.weight"], weights[f"{name}.scales"], weights[f"{name}.biases"]
    except KeyError as exc:
        raise CheckpointError(f"missing quantised tensor {exc.args[0]!r}") from exc
    if w.dtype not in (torch.uint32, torch.int32) or s.dtype != torch.bfloat16 or b.dtype != torch.bfloat16:
        raise CheckpointError(f"{name}: expected uint32 codes and bf16 scales/biases, got {w.dtype}, {s.dtype}")
    if s.shape != b.shape or w.shape[0] != s.shape[0] or w.shape[1] * 8 != s.shape[1] * 64:
        raise CheckpointError(f"{name}: inconsistent shapes {tuple(w.shape)}, {tuple(s.shape)}, {tuple(b.shape)}")
    return w.view(torch.int32), s, b


def _norm(weights: dict, name: str) -> torch.Tensor:
    t = weights.get(f"{name}.weight")
    if t is None:
        raise CheckpointError(f"missing norm {name!r}")
    return t.to(torch.bfloat16)


def _rows(q, r0: int, r1: int):
    return tuple(t[r0:r1] for t in q)


def _cols(q, c0: int, c1: int):
    w, s, b = q
    return w[:, c0 // 8:c1 // 8], s[:, c0 // 64:c1 // 64], b[:, c0 // 64:c1 // 64]


def _cat(*qs):
    return tuple(torch.cat([q[i] for q in qs]) for i in range(3))


def assign_weights(model: QuantModel, weights: dict) -> None:
    """Fill `model` (its config, tensor-parallel rank and device already set) from MLX-named 4-bit tensors."""
    c, tp, dev = model.cfg, model.tp, model.device
    sh = tp_shard(c, tp, model.rank)
    gemma = c.family == "gemma3"

    def lin(q, packed: bool = True) -> Linear4:
        w, s, b = (t.contiguous().to(dev) for t in q)
        return Linear4(w, s, b, kernels.Packed(w, s, b) if packed else None)

    def check(q, n: int, k: int, name: str):
        if tuple(q[0].shape) != (n, k // 8):
            raise CheckpointError(f"{name}: shape {tuple(q[0].shape)}, expected ({n}, {k // 8}) for the config")
        return q

    emb = check(_q(weights, "model.embed_tokens"), c.vocab, c.hidden, "embed_tokens")
    head_q = _q(weights, "lm_head") if "lm_head.weight" in weights else emb
    check(head_q, c.vocab, c.hidden, "lm_head")
    tied = head_q is emb
    if tp == 1:
        model.embed = lin(emb, packed=tied)
        model.head = model.embed if tied else lin(head_q)
    else:
        model.embed = lin(emb, packed=False)  # the gather reads the whole table; the head is this rank's slice
        model.head = lin(_rows(head_q, *sh["vocab"]))
    d = c.head_dim
    model.layers = []
    for i in range(c.layers):
        pre = f"model.layers.{i}"
        q = check(_q(weights, f"{pre}.self_attn.q_proj"), c.heads * d, c.hidden, "q_proj")
        k = check(_q(weights, f"{pre}.self_attn.k_proj"), c.kv_heads * d, c.hidden, "k_proj")
        v = check(_q(weights, f"{pre}.self_attn.v_proj"), c.kv_heads * d, c.hidden, "v_proj")
        o = check(_q(weights, f"{pre}.self_attn.o_proj"), c.hidden, c.heads * d, "o_proj")
        gate = check(_q(weights, f"{pre}.mlp.gate_proj"), c.inter, c.hidden, "gate_proj")
        up = check(_q(weights, f"{pre}.mlp.up_proj"), c.inter, c.hidden, "up_proj")
        down = check(_q(weights, f"{pre}.mlp.down_proj"), c.hidden, c.inter, "down_proj")
        if tp > 1:
            q, k, v = (_rows(x, a - off, e - off) for x, (a, e), off in
                       ((q, sh["q"], 0), (k, sh["k"], c.heads * d), (v, sh["v"], (c.heads + c.kv_heads) * d)))
            o = _cols(o, *sh["o_cols"])
            gate, up = _rows(gate, *sh["inter"]), _rows(up, *sh["inter"])
            down = _cols(down, *sh["inter"])
        gate_up = tuple(interleave_gate_up(g.contiguous(), u.contiguous()) for g, u in zip(gate, up))
        layer = Layer(lin(_cat(q, k, v)), lin(o), lin(gate_up), lin(down),
                      _norm(weights, f"{pre}.input_layernorm").to(dev),
                      _norm(weights, f"{pre}.pre_feedforward_layernorm" if gemma
                            else f"{pre}.post_attention_layernorm").to(dev),
                      _norm(weights, f"{pre}.self_attn.q_norm").to(dev),
                      _norm(weights, f"{pre}.self_attn.k_norm").to(dev))
        if gemma:
            layer.post_attn_norm = _norm(weights, f"{pre}.post_attention_layernorm").to(dev)
            layer.post_ff_norm = _norm(weights, f"{pre}.post_feedforward_layernorm").to(dev)
        model.layers.append(layer)
    model.final_norm = _norm(weights, "model.norm").to(dev)


def load_mlx_4bit(root: str | Path, device: torch.device | str = "cuda", **model_kwargs) -> QuantModel:
    """A `QuantModel` from an MLX 4-bit snapshot directory (config.json + *.safetensors). `model_kwargs` are
    QuantModel's (max_seqs, max_ctx, max_rows, max_logit_rows, tp, rank, group, ...)."""
    root = Path(root).expanduser()
    try:
        config = json.loads((root / "config.json").read_text(encoding="utf-8"))
    except (OSError, UnicodeError, json.JSONDecodeError) as exc:
        raise CheckpointError(f"{root}: unreadable config.json ({exc})") from exc
    if not isinstance(config, dict):
        raise CheckpointError("config.json root must be an object")
    quantisation(config)
    cfg = model_config(config, name=root.name)
    return QuantModel(cfg, device, weights=read_tensors(root), **model_kwargs)


# ---- writing ------------------------------------------------------------------------------------------------
def _deinterleave(t: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    rows = t.shape[0] // 2
    blocks = t.reshape(rows // 16, 2, 16, *t.shape[1:])
    return blocks[:, 0].reshape(rows, *t.shape[1:]), blocks[:, 1].reshape(rows, *t.shape[1:])


def save_mlx_4bit(model: QuantModel, root: str | Path) -> Path:
    """Write a single-GPU `QuantModel` as an MLX 4-bit snapshot (config.json + model.safetensors)."""
    from safetensors.torch import save_file

    if model.tp != 1:
        raise CheckpointError("save a tensor-parallel model from its tp = 1 counterpart")
    c = model.cfg
    root = Path(root)
    root.mkdir(parents=True, exist_ok=True)
    out: dict[str, torch.Tensor] = {}

    def put(name: str, w, s, b) -> None:
        out[f"{name}.weight"] = w.contiguous().cpu().view(torch.uint32)
        out[f"{name}.scales"] = s.contiguous().cpu()
        out[f"{name}.biases"] = b.contiguous().cpu()

    put("model.embed_tokens", model.embed.w, model.embed.s, model.embed.b)
    if model.head is not model.embed:
        put("lm_head", model.head.w, model.head.s, model.head.b)
    d = c.head_dim
    bounds = [0, c.heads * d, (c.heads + c.kv_heads) * d, c.qkv_rows]
    for i, layer in enumerate(model.layers):
        pre = f"model.layers.{i}"
        for j, part in enumerate(("q_proj", "k_proj", "v_proj")):
            r0, r1 = bounds[j], bounds[j + 1]
            put(f"{pre}.self_attn.{part}", layer.qkv.w[r0:r1], layer.qkv.s[r0:r1], layer.qkv.b[r0:r1])
        put(f"{pre}.self_attn.o_proj", layer.o.w, layer.o.s, layer.o.b)
        (gw, uw), (gs, us), (gb, ub) = (_deinterleave(t) for t in (layer.gate_up.w, layer.gate_up.s, layer.gate_up.b))
        put(f"{pre}.mlp.gate_proj", gw, gs, gb)
        put(f"{pre}.mlp.up_proj", uw, us, ub)
        put(f"{pre}.mlp.down_proj", layer.down.w, layer.down.s, layer.down.b)
        out[f"{pre}.input_layernorm.weight"] = layer.in_norm.cpu()
        out[f"{pre}.self_attn.q_norm.weight"] = layer.q_norm.cpu()
        out[f"{pre}.self_attn.k_norm.weight"] = layer.k_norm.cpu()
        if c.family == "gemma3":
            out[f"{pre}.pre_feedforward_layernorm.weight"] = layer.post_norm.cpu()
            out[f"{pre}.post_attention_layernorm.weight"] = layer.post_attn_norm.cpu()
            out[f"{pre}.post_feedforward_layernorm.weight"] = layer.post_ff_norm.cpu()
        else:
            out[f"{pre}.post_attention_layernorm.weight"] = layer.post_norm.cpu()
    out["model.norm.weight"] = model.final_norm.cpu()
    save_file(out, str(root / "model.safetensors"))
    config = {"model_type": "gemma3_text" if c.family == "gemma3" else "qwen3", "hidden_size": c.hidden,
              "num_hidden_layers": c.layers, "num_attention_heads": c.heads, "num_key_value_heads": c.kv_heads,
              "head_dim": d, "intermediate_size": c.inter, "vocab_size": c.vocab, "rope_theta": c.rope_theta,
              "rms_norm_eps": c.eps, "tie_word_embeddings": model.head is model.embed,
              "quantization": {"group_size": 64, "bits": 4}}
    if c.rope_scale != 1.0:
        config["rope_scaling"] = {"rope_type": "linear", "factor": c.rope_scale}
    if c.family == "gemma3":
        config.update(sliding_window=c.sliding_window, sliding_window_pattern=c.global_every,
                      rope_local_base_freq=c.rope_local_theta, query_pre_attn_scalar=round(c.scale ** -2))
    (root / "config.json").write_text(json.dumps(config, indent=1))
    return root
