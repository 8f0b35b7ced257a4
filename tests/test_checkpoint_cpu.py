"""MLX 4-bit snapshot handling on the CPU: config.json parsing (Qwen3, Gemma-3 text and multimodal forms, linear
RoPE scaling), the quantisation checks the reference applies (ironmule/model_identity.py:201-212) narrowed to
4-bit groups of 64, tensor names with a multimodal prefix, and the gate/up interleave round trip."""
from __future__ import annotations

import json

import pytest
import torch

from ironmule_b200 import checkpoint
from ironmule_b200.engine import PRESETS, interleave_gate_up

QWEN3_4B = {"model_type": "qwen3", "hidden_size": 2560, "num_hidden_layers": 36, "num_attention_heads": 32,
            "num_key_value_heads": 8, "head_dim": 128, "intermediate_size": 9728, "vocab_size": 151936,
            "rope_theta": 1000000, "rms_norm_eps": 1e-06, "tie_word_embeddings": True,
            "quantization": {"group_size": 64, "bits": 4}}
GEMMA3_12B = {"model_type": "gemma3", "quantization": {"group_size": 64, "bits": 4},
              "text_config": {"model_type": "gemma3_text", "hidden_size": 3840, "num_hidden_layers": 48,
                              "num_attention_heads": 16, "num_key_value_heads": 8, "head_dim": 256,
                              "intermediate_size": 15360, "vocab_size": 262144, "sliding_window": 1024,
                              "sliding_window_pattern": 6, "rope_local_base_freq": 10000.0,
                              "rope_theta": 1000000.0, "query_pre_attn_scalar": 256,
                              "rope_scaling": {"rope_type": "linear", "factor": 8.0}}}


def test_qwen3_config_matches_the_preset():
    cfg = checkpoint.model_config(QWEN3_4B, "qwen3-4b")
    assert cfg == PRESETS["qwen3-4b"]


def test_gemma3_multimodal_config():
    cfg = checkpoint.model_config(GEMMA3_12B, "gemma3-12b")
    assert cfg.family == "gemma3" and cfg.hidden == 3840 and cfg.layers == 48 and cfg.head_dim == 256
    assert cfg.sliding_window == 1024 and cfg.global_every == 6 and cfg.rope_scale == 8.0
    assert cfg.scale == 256 ** -0.5 and cfg.vocab == 262144
    assert cfg == PRESETS["gemma3-12b"].__class__(**{**PRESETS["gemma3-12b"].__dict__, "rope_scale": 8.0})


@pytest.mark.parametrize("change,match", [
    ({"quantization": {"group_size": 64, "bits": 8}}, "4-bit"),
    ({"quantization": {"group_size": 32, "bits": 4}}, "groups of 64"),
    ({"quantization": {"group_size": True, "bits": 4}}, "positive integer"),
    ({"quantization": None}, "no quantization"),
])
def test_quantisation_checks(change, match):
    with pytest.raises(checkpoint.CheckpointError, match=match):
        checkpoint.quantisation({**QWEN3_4B, **change})


@pytest.mark.parametrize("change,match", [
    ({"model_type": "llama"}, "qwen3 and gemma3"),
    ({"model_type": ""}, "no model_type"),
    ({"head_dim": 64}, "head_dim"),
    ({"rope_scaling": {"rope_type": "yarn", "factor": 4.0}}, "linear only"),
])
def test_unsupported_configs_are_refused(change, match):
    with pytest.raises(checkpoint.CheckpointError, match=match):
        checkpoint.model_config({**QWEN3_4B, **change})


def test_tensor_names_lose_the_multimodal_prefix(tmp_path):
    from safetensors.torch import save_file

    save_file({"language_model.model.norm.weight": torch.ones(4, dtype=torch.bfloat16),
               "lm_head.weight": torch.zeros((2, 1), dtype=torch.uint32)}, str(tmp_path / "a.safetensors"))
    t = checkpoint.read_tensors(tmp_path)
    assert set(t) == {"model.norm.weight", "lm_head.weight"} and t["lm_head.weight"].dtype == torch.uint32


def test_missing_snapshot_pieces(tmp_path):
    with pytest.raises(checkpoint.CheckpointError, match="config.json"):
        checkpoint.load_mlx_4bit(tmp_path, device="cpu")
    (tmp_path / "config.json").write_text(json.dumps(QWEN3_4B))
    with pytest.raises(checkpoint.CheckpointError, match="no safetensors"):
        checkpoint.read_tensors(tmp_path)


def test_gate_up_interleave_round_trip():
    g = torch.arange(64 * 3, dtype=torch.int32).reshape(64, 3)
    u = -g
    gu = interleave_gate_up(g, u)
    g2, u2 = checkpoint._deinterleave(gu)
    assert torch.equal(g2, g) and torch.equal(u2, u)


def test_shard_slices_of_quantised_tensors_equal_quantised_shards():
    """The loader cuts tensor-parallel shards out of the quantised tensors (rows for q/k/v/gate/up/vocabulary,
    64-aligned columns for o/down). Quantisation is per row and per 64-wide group, so a slice of the quantised
    tensor equals the quantisation of the same slice of the dense matrix (oracle quantiser)."""
    import numpy as np

    from oracle import bf16, quant

    rng = np.random.default_rng(0)
    w = bf16.round_f32(rng.normal(0, 0.05, (96, 512)).astype(np.float32))
    wq, s, b = quant.quantize(w)
    as_torch = (torch.from_numpy(wq.view(np.int32)), torch.from_numpy(s.view(np.int16)),
                torch.from_numpy(b.view(np.int16)))
    for r0, r1 in ((0, 32), (32, 96)):
        want = quant.quantize(w[r0:r1])
        got = checkpoint._rows(as_torch, r0, r1)
        for g, x in zip(got, want):
            assert np.array_equal(g.numpy(), x.view(g.numpy().dtype))
    for c0, c1 in ((0, 256), (256, 512), (128, 384)):
        want = quant.quantize(np.ascontiguousarray(w[:, c0:c1]))
        got = checkpoint._cols(as_torch, c0, c1)
        for g, x in zip(got, want):
            assert np.array_equal(g.contiguous().numpy(), x.view(g.numpy().dtype))
