"""Tensor parallelism on the CPU, two gloo ranks: each rank takes its engine.tp_shard slices of the same seeded
full matrices; the column shards (q, k, v, gate, up, head vocabulary) gathered in rank order, and the row-shard
partial products (o, down) all-reduced, reproduce the full model's products -- the sharding rules and the
collective steps of the tensor-parallel forward, without a GPU."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ironmule_b200 import engine

CFG = engine.ModelConfig("tp-test", 256, 1, 8, 4, 32, 512, 1024)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, world: int, port: int, failures) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        c = CFG
        g = torch.Generator().manual_seed(0)
        x = torch.randn(3, c.hidden, generator=g, dtype=torch.float64)
        qkv = torch.randn(c.qkv_rows, c.hidden, generator=g, dtype=torch.float64)
        o = torch.randn(c.hidden, c.heads * c.head_dim, generator=g, dtype=torch.float64)
        gate = torch.randn(c.inter, c.hidden, generator=g, dtype=torch.float64)
        down = torch.randn(c.hidden, c.inter, generator=g, dtype=torch.float64)
        head = torch.randn(c.vocab, c.hidden, generator=g, dtype=torch.float64)
        sh = engine.tp_shard(c, world, rank)
        cut = lambda a, key: a[slice(*sh[key])]  # noqa: E731

        def gathered(local):
            parts = [torch.empty_like(local) for _ in range(world)]
            dist.all_gather(parts, local.contiguous())
            return parts

        # column shards: each rank's q / k / v heads, gathered in rank order, are the full blocks
        full = x @ qkv.T
        for key, (lo, hi) in (("q", (0, c.heads * c.head_dim)),
                              ("k", (c.heads * c.head_dim, (c.heads + c.kv_heads) * c.head_dim)),
                              ("v", ((c.heads + c.kv_heads) * c.head_dim, c.qkv_rows))):
            assert torch.equal(torch.cat(gathered(x @ cut(qkv, key).T), dim=1), full[:, lo:hi]), key
        # row shard of o: the rank's heads' columns; partial products all-reduced = the full product
        attn = torch.randn(3, c.heads * c.head_dim, generator=torch.Generator().manual_seed(1), dtype=torch.float64)
        part = attn[:, slice(*sh["o_cols"])] @ o[:, slice(*sh["o_cols"])].T
        dist.all_reduce(part)
        assert torch.allclose(part, attn @ o.T, rtol=1e-12, atol=1e-9)
        # gate rows and down columns over the same intermediate slice
        act = torch.randn(3, c.inter, generator=torch.Generator().manual_seed(2), dtype=torch.float64)
        assert torch.equal(torch.cat(gathered(x @ cut(gate, "inter").T), dim=1), x @ gate.T)
        part = act[:, slice(*sh["inter"])] @ down[:, slice(*sh["inter"])].T
        dist.all_reduce(part)
        assert torch.allclose(part, act @ down.T, rtol=1e-12, atol=1e-9)
        # head: vocabulary slices gathered in rank order are the full logits (the engine's [tp][rows][V/tp] ->
        # [rows][V] permute)
        stacked = torch.stack(gathered(x @ cut(head, "vocab").T))  # [tp, rows, V/tp]
        assert torch.equal(stacked.permute(1, 0, 2).reshape(3, c.vocab), x @ head.T)
    except AssertionError as exc:
        failures.put(f"rank {rank}: {exc}")
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_tensor_parallel_shards_reproduce_the_full_products(world):
    ctx = mp.get_context("spawn")
    failures = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, failures)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert failures.empty()


def test_shards_cover_the_model_and_respect_groups():
    c = engine.PRESETS["gemma3-27b"]
    for tp in (2, 4, 8):
        shards = [engine.tp_shard(c, tp, r) for r in range(tp)]
        for key in ("o_cols", "inter", "vocab"):
            assert shards[0][key][0] == 0 and all(a[key][1] == b[key][0] for a, b in zip(shards, shards[1:]))
        assert shards[-1]["inter"][1] == c.inter and shards[-1]["vocab"][1] == c.vocab
        for s in shards:
            assert (s["o_cols"][1] - s["o_cols"][0]) % 64 == 0 and (s["inter"][1] - s["inter"][0]) % 64 == 0
