"""MLX 4-bit snapshots on the device: a model written with save_mlx_4bit and read back with load_mlx_4bit gives
the same logits bit for bit (Qwen3 and Gemma-3 forms, tied and separate heads), and greedy decoding from the
loaded snapshot returns the original model's tokens."""
from __future__ import annotations

import pytest
import torch

from ironmule_b200 import checkpoint, engine, kernels

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name,tied", [("tiny-target", True), ("tiny-target", False), ("tiny-gemma", True)])
def test_snapshot_round_trip_changes_no_bits(cuda, tmp_path, name, tied):
    model = engine.QuantModel(engine.PRESETS[name], "cuda", seed=3, sigma=0.08, max_ctx=256)
    if not tied:
        gen = torch.Generator(device="cuda").manual_seed(11)
        table = (torch.randn((model.cfg.vocab, model.cfg.hidden), generator=gen, device="cuda") * 0.08)
        wq, s, b = kernels.quantize(table.to(torch.bfloat16))
        model.head = engine.Linear4(wq, s, b, kernels.Packed(wq, s, b))
    root = checkpoint.save_mlx_4bit(model, tmp_path / name)
    loaded = checkpoint.load_mlx_4bit(root, "cuda", max_ctx=256)
    assert (loaded.head is loaded.embed) == tied
    prompt = torch.randint(0, 1000, (20,), generator=torch.Generator().manual_seed(1)).to(torch.int32).to(cuda)
    a = model.logits_for(prompt, 0).clone()
    b2 = loaded.logits_for(prompt, 0)
    assert torch.equal(a.view(torch.int16), b2.view(torch.int16))
    model2 = checkpoint.load_mlx_4bit(root, "cuda", max_ctx=256)
    model.k_cache.zero_()
    model.v_cache.zero_()
    assert engine.greedy_decode(model2, prompt, 12) == engine.greedy_decode(model, prompt, 12)
