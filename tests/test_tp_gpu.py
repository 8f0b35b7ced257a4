"""Tensor parallelism on 2 GPUs (NCCL, one process per GPU; skipped with fewer GPUs). The tp = 2 forward
agrees with the tp = 1 model of the same seed within the forward tolerance (the bf16 all-reduce of partial
projections rounds where one GPU's qGEMM would not), and speculative decoding on the tensor-parallel target
returns exactly the tensor-parallel model's own greedy tokens: with two ranks a partial sum is a single
commutative add, so every row is still computed the same way however many rows share the call."""
from __future__ import annotations

import datetime
import os
import socket
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, world: int, port: int, failures, tmp: str) -> None:
    import torch.distributed as dist

    from ironmule_b200 import engine

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        for name in ("tiny-target", "tiny-gemma"):
            model = engine.QuantModel(engine.PRESETS[name], dev, seed=4, sigma=0.08, max_ctx=256, tp=world,
                                      rank=rank, group=dist.group.WORLD)
            prompt = torch.randint(0, 1000, (24,), generator=torch.Generator().manual_seed(2)).to(torch.int32).to(dev)
            got = model.logits_for(prompt, 0).float().cpu().numpy()
            ref = engine.QuantModel(engine.PRESETS[name], dev, seed=4, sigma=0.08, max_ctx=256)
            want = ref.logits_for(prompt, 0).float().cpu().numpy()
            err = np.abs(got - want).max()
            assert err <= 2e-2 * np.abs(want).max(), (name, err)
            assert np.mean(got.argmax(1) == want.argmax(1)) >= 0.9, name
            # the tp = 1 model written as an MLX 4-bit snapshot and read back with tp = 2: the same shards
            from ironmule_b200 import checkpoint
            root = checkpoint.save_mlx_4bit(ref, Path(tmp) / f"{name}-{rank}")
            loaded = checkpoint.load_mlx_4bit(root, dev, max_ctx=256, tp=world, rank=rank, group=dist.group.WORLD)
            again = loaded.logits_for(prompt, 0).float().cpu().numpy()
            assert np.array_equal(again, got), name
            del ref, loaded
            # speculation on the tensor-parallel target == its own greedy decoding (draft replicated)
            fresh = engine.QuantModel(engine.PRESETS[name], dev, seed=4, sigma=0.08, max_ctx=256, tp=world, rank=rank,
                                      group=dist.group.WORLD)
            plain = engine.greedy_decode(fresh, prompt, 20)
            draft_name = "tiny-draft" if name == "tiny-target" else "tiny-gemma"
            draft = engine.QuantModel(engine.PRESETS[draft_name], dev, seed=7, sigma=0.08, max_ctx=256)
            dec = engine.SpecDecoder(model, draft, k=4)
            dec.start([prompt], max_new=20)
            dec.round()
            dec.capture()
            while not dec.done():
                dec.run_rounds(2)
            assert dec.generated(0, prompt.numel()) == plain, name
            dec.graph = None
            torch.cuda.synchronize()
        dist.barrier()
    except AssertionError as exc:
        failures.put(f"rank {rank}: {exc}")
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tensor_parallel_forward_and_speculation_on_two_gpus(tmp_path):
    ctx = torch.multiprocessing.get_context("spawn")
    failures = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, failures, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
    for p in procs:
        if p.is_alive():
            p.kill()
    msgs = []
    while not failures.empty():
        msgs.append(failures.get())
    assert all(p.exitcode == 0 for p in procs), ([p.exitcode for p in procs], msgs)
