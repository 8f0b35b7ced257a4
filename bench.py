#!/usr/bin/env python
"""Benchmark of the speculative-decoding hot path on B200 (one JSON line on rank 0).

Workload (default, BASELINE config "end-to-end greedy speculative decoding, batch 1"): Qwen3-4B-shaped target
(36 layers, hidden 2560, 32/8 heads, head_dim 128, SwiGLU 9728, vocab 151936, tied embeddings) and
Qwen3-0.6B-shaped draft (28 layers, hidden 1024, 16/8 heads, SwiGLU 3072), both random-init and quantised to
MLX-affine 4-bit group 64 on the device; k = 4 drafts; a 512-token prompt of uniform random ids (seed 0 +
rank); greedy acceptance. A step is one speculative round (4 draft passes + 1 verify pass + accept); `value`
is committed tokens per second over all ranks (replicas, one independent sequence per GPU; no collective on
the data path), timed with CUDA events over K rounds replayed from one captured CUDA graph. Every round
streams the full 3.6 GB of weights, far more than the 126 MB L2, so no flush is needed.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload spec_decode|verify_step|qgemm_pass|stochastic|tree|tp|attention|kquant|
                                small_kernels|prefill]

--workload stochastic: BASELINE config 3's round -- Qwen3-4B + 0.6B, temperature 0.7, top-p 0.95, k = 4, rejection
sampling with residual resampling on Philox -- over 32 concurrent sequences with prompt lengths drawn uniformly
from [128, 2048] (seed 0): 32 x 5 = 160 verify rows per qGEMM call. --workload tree: config 4's tree verification
on Gemma-3-12B shapes (48 layers, hidden 3840, 16/8 heads, head_dim 256, GeGLU 15360, vocab 262144) with a
Gemma-3-1B-shaped draft, a 4 x 2 x 2 draft tree verified as root + 28 nodes = 29 rows per sequence, 8 sequences,
1024-token prompts. --workload tp (under torchrun, N ranks): config 5a -- Gemma-3-27B shapes tensor-parallel over
the N GPUs (NCCL all-reduce after o and down, all-gathered vocabulary-sharded head) with a replicated
Gemma-3-1B-shaped draft, greedy, k = 4, 64 sequences with 512-token prompts; one job over all ranks, so `value` is
that job's tokens/s (strong scaling).

--impl reference times the CPU implementation of the same round (the oracle port in oracle/spec.py: the
reference's greedy round with projections dequantised and dotted in float32 by OpenMP C code) on the box's host
cores; rank 0 alone runs it under torchrun.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

K_DRAFTS = 4
PROMPT = 512
NEW_TOKENS = 256
MAX_CTX = 1536


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["spec_decode", "verify_step", "qgemm_pass", "stochastic", "tree", "tp",
                                           "attention", "kquant", "small_kernels", "prefill"],
                    default="spec_decode")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-tp", action="store_true", help="default workload: skip the tensor-parallel config-5a record")
    ap.add_argument("--rows", type=int, default=0,
                    help="verify_step: activation rows of the qGEMM (default 5); attention: rows per sequence (5)")
    ap.add_argument("--attn-case", choices=["config3-verify", "config3-draft", "config2-draft"],
                    default="config3-verify",
                    help="attention: config 3's verify (32 sequences, Qwen3-4B heads, 5 rows) or draft pass "
                         "(Qwen3-0.6B heads, 1 row), or config 2's draft pass (1 sequence, 520 keys)")
    ap.add_argument("--kpc", type=int, default=64, help="attention: keys per split (a multiple of 64)")
    ap.add_argument("--layers", type=int, default=0, help="kquant: layers of Q4_K matrices (default 36)")
    ap.add_argument("--qgemm-path", type=int, choices=[0, 1, 2], default=0,
                    help="packed qGEMM kernel: 0 automatic, 1 warp MMA only, 2 tcgen05 tensor cores only (same bits)")
    return ap.parse_args()


def peaks() -> dict:
    """HBM GB/s and dense bf16 TFLOP/s (burst) measured on this pool, else the recorded fallback figures."""
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d.get("bf16_tflops", 1590.0)),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


class Clocks:
    """nvidia-smi samples (every 50 ms) of the SM clock and throttle reasons, started before the warm-up steps and
    stopped after the timed region, so that the samples under load cover the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index, self.proc, self.out = index, None, ""

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.1)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(args):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def reduce_max(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def reduce_sum(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ---- CPU side (oracle port): the reported baseline and the --impl reference arm ---------------------------
def cpu_round_rate(rounds: int, warmup: int, prompt_len: int = 16, threads: int | None = None) -> dict:
    """Committed tokens/s of the CPU port of the round on random-weight models of the benchmark's shapes."""
    if threads:
        os.environ["OMP_NUM_THREADS"] = str(threads)
    from ironmule_b200.engine import PRESETS
    from oracle.spec import CpuSpecDecoder, random_model

    import numpy as np

    slots = prompt_len + (rounds + warmup + 2) * (K_DRAFTS + 1) + 8
    target = random_model(PRESETS["qwen3-4b"], seed=0, slots=slots)
    draft = random_model(PRESETS["qwen3-0.6b"], seed=1, slots=slots)
    dec = CpuSpecDecoder(target, draft, k=K_DRAFTS, slots=slots)
    prompt = np.random.default_rng(0).integers(0, 151936, prompt_len).tolist()
    dec.start(prompt)
    for _ in range(warmup):
        dec.round()
    made = 0
    t0 = time.perf_counter()
    for _ in range(rounds):
        made += len(dec.round())
    sec = time.perf_counter() - t0
    return {"value": made / sec, "seconds": sec, "rounds": rounds, "tokens": made}


def cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def run_reference(args, world: int, rank: int) -> None:
    if rank != 0:
        return
    n = cores()
    res = cpu_round_rate(args.steps, args.warmup, threads=n)
    sample = (f"{args.steps} rounds after {args.warmup} warm-up rounds, 16-token prompt, Qwen3-4B/0.6B shapes with "
              f"random 4-bit weights, k=4 greedy, OpenMP dequantise-and-dot projections on {n} threads")
    line = {"impl": "reference", "metric": "accepted tokens/s (spec decode, Qwen3-4B + 0.6B draft, k=4, batch 1)",
            "value": round(res["value"], 4), "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(1000 * res["seconds"] / args.steps, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16 activations, 4-bit weights",
            "data": "synthetic (random weights and prompt)",
            "config": {"workload": "config 2: greedy spec decode Qwen3-4B target + Qwen3-0.6B draft, k=4, batch 1",
                       "cpu_path": "oracle port (the reference's CPU paths, MLX CPU and llama.cpp, are not installed)"},
            "cpu_baseline": {"value": round(res["value"], 4), "unit": "tokens/s", "cores": n, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(res["value"], 4), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---- GPU side --------------------------------------------------------------------------------------------
# DRAM bytes (read + write) per launch of the verify pass's packed qGEMMs, the mean over the pass's 145 launches
# from one ncu capture of `python bench.py --workload qgemm_pass` (the command and the per-kernel figures are in
# the profile named below). Re-captured whenever the kernel changes.
VERIFY_PASS_DRAM_BYTES_PER_LAUNCH = 15_720_992
VERIFY_PASS_DRAM_SOURCE = "profiles/qgemm_packed_verify_pass_traffic.md (ncu, 145 launches, one B200)"


def qgemm_roofline(target, peak_gbs: float, reps: int = 20) -> dict:
    """The dominant kernel: every packed qGEMM of one verify pass (M = k+1 = 5 rows: 36 x [qkv, o, gate_up,
    down] and the head), launched as the forward launches them (RMSNorm prologues on qkv / gate_up / head,
    residual + sums-of-squares epilogues on o / down), captured once as a graph and replayed; CUDA events on
    the launching stream give the mean launch duration and the achieved bandwidth over the algorithmic bytes
    (4-bit weights at 0.5625 B per weight + activations in + results out)."""
    import torch

    from ironmule_b200 import kernels

    m = K_DRAFTS + 1
    c = target.cfg
    x = torch.randn((m, max(c.inter, c.heads * c.head_dim, c.hidden)), device=target.device).to(torch.bfloat16)
    res = torch.randn((m, c.hidden), device=target.device).to(torch.bfloat16)
    out = torch.zeros((m, c.vocab), dtype=torch.bfloat16, device=target.device)
    sq = torch.ones((target.h_tiles, 32), dtype=torch.float32, device=target.device)
    calls, total_bytes = [], 0

    def add(lin, epi, norm):
        nonlocal total_bytes
        n_out = lin.n // 2 if epi == "swiglu" else lin.n
        calls.append((lin, epi, norm))
        total_bytes += lin.n * lin.k * 9 // 16 + m * lin.k * 2 + m * n_out * 2 + (m * lin.n * 2 if epi == "residual" else 0)

    for layer in target.layers:
        add(layer.qkv, "store", layer.in_norm)
        add(layer.o, "residual", None)
        add(layer.gate_up, "swiglu", layer.post_norm)
        add(layer.down, "residual", None)
    add(target.embed, "store", target.final_norm)

    def run():
        for lin, epi, norm in calls:
            xin = res if norm is not None else x.view(-1)[: m * lin.k].view(m, lin.k)
            kernels.qgemm_packed(xin, lin.p, epilogue=epi, residual=res if epi == "residual" else None,
                                 out=res if epi == "residual" else out, ws=target.ws_gemm,
                                 norm_sq=sq if norm is not None else None, norm_parts=target.h_tiles,
                                 norm_weight=norm, eps=c.eps, out_sq=sq if epi == "residual" else None)

    run()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        run()
    g.replay()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    sec = e0.elapsed_time(e1) / 1000 / reps
    launches = len(calls)
    achieved = total_bytes / sec / 1e9
    return {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak_gbs, "unit": "GB/s",
            "frac": round(achieved / peak_gbs, 4), "traffic": VERIFY_PASS_DRAM_BYTES_PER_LAUNCH,
            "traffic_source": VERIFY_PASS_DRAM_SOURCE,
            "kernel": "qgemm_packed_kernel (all 145 qGEMMs of one Qwen3-4B verify pass, M=5)",
            "launches": launches, "us_per_launch": round(sec / launches * 1e6, 2),
            "algorithmic_bytes_per_launch": total_bytes // launches, "pass_us": round(sec * 1e6, 1)}


def run_spec_decode(args, world: int, rank: int, local: int) -> None:
    import torch

    from ironmule_b200.engine import PRESETS, QuantModel, SpecDecoder

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    pk = peaks()
    target = QuantModel(PRESETS["qwen3-4b"], device, seed=0, max_ctx=MAX_CTX, max_rows=256, max_logit_rows=8)
    draft = QuantModel(PRESETS["qwen3-0.6b"], device, seed=1, max_ctx=MAX_CTX, max_rows=256, max_logit_rows=8)
    dec = SpecDecoder(target, draft, k=K_DRAFTS, batch=1)
    gen = torch.Generator().manual_seed(rank)
    prompt = torch.randint(0, PRESETS["qwen3-4b"].vocab, (PROMPT,), generator=gen, dtype=torch.int32)

    # ---- device-timed rounds from the captured graph
    room = MAX_CTX - PROMPT - K_DRAFTS - 8
    dec.start([prompt.to(device)], max_new=room)
    dec.round()
    torch.cuda.synchronize()
    dec.capture()
    clocks = Clocks(local)
    clocks.start()
    dec.run_rounds(args.warmup)
    torch.cuda.synchronize()
    before = dec.read_stats()
    stream = torch.cuda.current_stream(device)
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("timed_rounds")
    e0.record(stream)
    dec.run_rounds(args.steps)
    e1.record(stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    after = dec.read_stats()
    tokens = after.tokens - before.tokens
    accepted = after.accepted - before.accepted
    if after.tokens - before.tokens < args.steps:
        print(f"warning: the sequence hit its length limit during timing ({tokens} tokens in {args.steps} rounds)",
              file=sys.stderr)
    max_ms = reduce_max(ms, world)
    total_tokens = reduce_sum(float(tokens), world)
    value = total_tokens / (max_ms / 1000)

    roof = qgemm_roofline(target, pk["hbm_gbs"])
    round_bytes = K_DRAFTS * draft.cfg.weight_bytes() + target.cfg.weight_bytes()

    # ---- end to end through the public streaming API (host prompt in, every round's tokens read back)
    e2e = None
    if not args.no_e2e:
        dec.generate([prompt.tolist()], 8)  # warm
        torch.cuda.synchronize()
        barrier(world)
        t0 = time.perf_counter()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        out = dec.generate([prompt.tolist()], NEW_TOKENS)
        s1.record(stream)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        rounds = dec.read_stats().rounds
        e2e_ms = reduce_max(max(s0.elapsed_time(s1), wall * 1000), world)
        e2e_tokens = reduce_sum(float(len(out[0])), world)
        e2e = {"value": round(e2e_tokens / (e2e_ms / 1000), 3), "unit": "tokens/s",
               "h2d_bytes_per_step": round(PROMPT * 4 / max(rounds, 1), 2),
               "d2h_bytes_per_step": 4 + 4 * (K_DRAFTS + 1),
               "what": f"generate(): {PROMPT}-token host prompt -> prefill both models -> {NEW_TOKENS} new tokens, "
                       f"each round's tokens copied to pinned host memory and handed to the caller",
               "rounds": rounds}

    tp = None
    if not args.no_tp:
        tp = tp_record(world, rank, local)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        n = cores()
        res = cpu_round_rate(rounds=3, warmup=1, threads=n)
        cpu = {"value": round(res["value"], 4), "unit": "tokens/s", "cores": n, "kind": "port",
               "sample": "3 speculative rounds (after 1 warm-up) on a 16-token prompt, Qwen3-4B/0.6B shapes, "
                         "random 4-bit weights, k=4 greedy; oracle port with OpenMP dequantise-and-dot projections"}

    if rank == 0:
        line = {
            "metric": "accepted tokens/s (spec decode, Qwen3-4B + 0.6B draft, k=4, batch 1)",
            "value": round(value, 3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(max_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16 activations, 4-bit weights (MLX affine g64)",
            "data": "synthetic (random-init weights, uniform random prompt)",
            "config": {"workload": "BASELINE config 2: greedy speculative decoding, Qwen3-4B target + Qwen3-0.6B "
                                   "draft, 4-bit affine g64, k=4, batch 1 per GPU, 512-token prompt",
                       "global_batch": world, "prompt": PROMPT, "k": K_DRAFTS,
                       "parallelism": f"replicas x{world}", "l2": "weights per round 3.6 GB >> 126 MB L2",
                       "accepted_per_round": round(accepted / args.steps, 4),
                       "round_weight_bytes": round_bytes,
                       "round_hbm_frac": round(round_bytes / (max_ms / args.steps / 1000) / 1e9 / pk["hbm_gbs"], 4)},
            "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "clocks": clk, "tp": tp,
            "gpu_launches": dec.launches_per_round() * args.steps,
            "peak_source": pk["source"]}
        print(json.dumps(line), flush=True)


def run_qgemm_pass(args, world: int, rank: int, local: int) -> None:
    """The dominant kernel alone: the 145 packed qGEMMs of one Qwen3-4B verify pass (M = 5), as the default
    workload's roofline measures them, on the target model only (2.3 GB of weights). The ncu capture of the
    pass's DRAM traffic runs this workload."""
    import torch

    from ironmule_b200.engine import PRESETS, QuantModel

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    pk = peaks()
    target = QuantModel(PRESETS["qwen3-4b"], device, seed=0, max_ctx=64, max_rows=32, max_logit_rows=8)
    roof = qgemm_roofline(target, pk["hbm_gbs"], reps=max(args.steps, 1))
    if rank == 0:
        line = {"metric": "qGEMM HBM GB/s (the 145 packed qGEMMs of one Qwen3-4B verify pass, M=5)",
                "value": roof["achieved"], "unit": "GB/s", "n_gpus": world, "steps": max(args.steps, 1),
                "warmup": 2, "ms_per_step": round(roof["pass_us"] / 1000, 4), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "bf16/4-bit", "data": "synthetic",
                "config": {"workload": "verify pass qGEMMs, Qwen3-4B, M=5, graph-replayed",
                           "l2": "2.26 GB of weights per pass >> 126 MB L2"},
                "roofline": roof, "peak_source": pk["source"]}
        print(json.dumps(line), flush=True)


def run_prefill(args, world: int, rank: int, local: int) -> None:
    """The e2e path's prompt prefill: the default workload's 511 prompt tokens (all but the last) into both
    models, in the chunks QuantModel.prefill cuts (256 rows per forward). Each step prefills both models from
    scratch; the timed steps run inside an NVTX range "timed" (the ncu launch list selects it)."""
    import torch

    from ironmule_b200.engine import PRESETS, QuantModel

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    target = QuantModel(PRESETS["qwen3-4b"], device, seed=0, max_ctx=MAX_CTX, max_rows=256, max_logit_rows=8)
    draft = QuantModel(PRESETS["qwen3-0.6b"], device, seed=1, max_ctx=MAX_CTX, max_rows=256, max_logit_rows=8)
    gen = torch.Generator().manual_seed(rank)
    prompt = torch.randint(0, PRESETS["qwen3-4b"].vocab, (PROMPT - 1,), generator=gen, dtype=torch.int32).to(device)
    steps = max(args.steps, 1)
    for _ in range(max(args.warmup, 1)):
        target.prefill(prompt)
        draft.prefill(prompt)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("timed")
    e0.record()
    for _ in range(steps):
        target.prefill(prompt)
        draft.prefill(prompt)
    e1.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    if rank == 0:
        line = {"metric": "prefill tokens/s (Qwen3-4B + Qwen3-0.6B, 511-token prompt)",
                "value": round((PROMPT - 1) / (ms / 1000), 1), "unit": "tokens/s", "n_gpus": world, "steps": steps,
                "warmup": max(args.warmup, 1), "ms_per_step": round(ms, 3), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "bf16 activations, 4-bit weights",
                "data": "synthetic", "config": {"workload": "prompt prefill of both models, 256-row chunks"}}
        print(json.dumps(line), flush=True)


def run_small_kernels(args, world: int, rank: int, local: int) -> None:
    """The kernels around the projections and attention, each alone through the entry point the engine calls, at
    the shapes of the configurations that launch them: greedy verification and the draft argmax (config 2), the
    stochastic acceptance and draft sampling (config 3: 32 sequences, k = 4, vocabulary 151,936), the tree's top-k
    (config 4: vocabulary 262,144) and bookkeeping, and the embedding gather. Inputs rotate over copies larger than
    the 126 MB L2 together; each kernel is timed from graph replays with CUDA events. Algorithmic bytes: the logits
    read once (2 B each), the embedding rows read once (0.5625 B per weight), the K/V a tree compaction moves."""
    import torch

    from ironmule_b200 import kernels

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    pk = peaks()
    gen = torch.Generator(device=device).manual_seed(0)
    stream = torch.cuda.current_stream(device)
    V, VG, K = 151936, 262144, K_DRAFTS
    bf = torch.bfloat16
    i32 = dict(dtype=torch.int32, device=device)

    def logits(rows, v, copies):
        return [(torch.randn((rows, v), generator=gen, device=device) * 2).to(bf) for _ in range(copies)]

    def timed(fn, copies, reps=64):
        for i in range(3):
            fn(i % copies)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(reps):
                fn(i % copies)
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(max(2, args.steps // reps)):
            g.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1000 / (max(2, args.steps // reps) * reps)  # us per call

    out = {}

    def record(name, us, nbytes, launches, what):
        gbs = nbytes / (us * 1e-6) / 1e9
        out[name] = {"us_per_call": round(us, 3), "algorithmic_bytes": int(nbytes), "gbs": round(gbs, 1),
                     "frac": round(gbs / pk["hbm_gbs"], 4), "launches_per_call": launches, "what": what}

    # config 2: greedy verification of 4 drafts (5 rows) and one draft row's argmax
    ver = logits(K + 1, V, 40)
    drafts = torch.randint(0, V, (K,), generator=gen, device=device, dtype=torch.int32)
    tok, cnt = torch.zeros((1, K + 1), **i32), torch.zeros((1,), **i32)
    ws_v = kernels.workspace(kernels.argmax_workspace_bytes(K + 1, V), device)
    record("verify_greedy", timed(lambda i: kernels.verify_greedy(ver[i], drafts, b=1, k=K, drafts_ld=K, tokens=tok,
                                                                  count=cnt, ws=ws_v), 40),
           (K + 1) * V * 2, 1, "argmax_kernel: 5 rows x 151,936 + greedy acceptance (config 2 verify)")
    one = logits(1, V, 200)
    pick = torch.zeros((1,), **i32)
    ws_1 = kernels.workspace(kernels.argmax_workspace_bytes(1, V), device)
    record("argmax_draft_row", timed(lambda i: kernels.argmax_rows(one[i], out=pick, ws=ws_1), 200), V * 2, 1,
           "argmax_kernel: 1 row x 151,936 (config 2 draft pick)")
    del ver, one
    # config 3: stochastic acceptance over 32 sequences x 5 rows and the draft sampling of 32 rows
    b = 32
    tl, dl = logits(b * (K + 1), V, 3), [x.view(K, b, V) for x in logits(K * b, V, 3)]
    dr = torch.randint(0, V, (b, K + 1), generator=gen, device=device, dtype=torch.int32)
    tok3, cnt3 = torch.zeros((b, K + 1), **i32), torch.zeros((b,), **i32)
    ws_a = kernels.workspace(kernels.sampling_workspace_bytes(b * (2 * K + 1)), device)
    off = torch.zeros((1,), dtype=torch.int64, device=device)
    record("accept_stochastic", timed(lambda i: kernels.accept_stochastic(
        tl[i], dl[i], dr[:, 1:], b=b, k=K, drafts_ld=K + 1, temperature=0.7, top_p=0.95, seed=0, offset_dev=off,
        tokens=tok3, count=cnt3, ws=ws_a), 3), (2 * K + 1) * b * V * 2, 3,
        "row_dist_kernel + accept_stochastic_kernel (+ residual resample): 32 x (5 target + 4 draft) rows x 151,936 "
        "(config 3)")
    ws_s = kernels.workspace(kernels.sampling_workspace_bytes(b), device)
    streams = torch.arange(b, **i32)
    smp = torch.zeros((b,), **i32)
    record("sample_rows", timed(lambda i: kernels.sample_rows(dl[i][0], 0.7, 0.95, 0, offset_dev=off, streams=streams,
                                                              draw=1000, out=smp, ws=ws_s), 3), b * V * 2, 2,
           "row_dist_kernel + sample_kernel: 32 draft rows x 151,936 (config 3 draft pick)")
    del tl, dl
    # config 4: top-k of the draft tree's levels (8 trees, 8 parents x 2 children at the widest level)
    rows_t = 8 * 8
    tk = logits(rows_t, VG, 5)
    kids = torch.zeros((rows_t * 2,), **i32)
    ws_t = kernels.workspace(kernels.topk_workspace_bytes(rows_t, VG, 4), device)
    record("topk_rows", timed(lambda i: kernels.topk_rows(tk[i], 2, out=kids, ws=ws_t), 5), rows_t * VG * 2, 1,
           "topk_kernel: 64 rows x 262,144, 2 children each (config 4 tree level)")
    del tk
    # the embedding gather of a verify pass (Qwen3-4B table, 5 rows) and of config 3's 160 rows
    from ironmule_b200.engine import PRESETS, QuantModel
    tgt = QuantModel(PRESETS["qwen3-4b"], device, seed=0, max_ctx=64, max_rows=160, max_logit_rows=8)
    ids = [torch.randint(0, V, (160,), generator=gen, device=device, dtype=torch.int32) for _ in range(16)]
    h = torch.zeros((160, 2560), dtype=bf, device=device)
    sq = torch.zeros((160,), dtype=torch.float32, device=device)
    for rows in (5, 160):
        record(f"embed_{rows}_rows", timed(lambda i: kernels.embed(ids[i], tgt.embed.w, tgt.embed.s, tgt.embed.b,
                                                                   out=h, rows=rows, out_sq=sq), 16),
               rows * 2560 * 9 // 16 + rows * 2560 * 2, 1, f"embed_kernel: {rows} rows of the 4-bit Qwen3-4B table")
    del tgt
    # config 4's tree bookkeeping: prepare, accept, compact over 8 trees of 4 x 2 x 2 (Gemma-3-12B caches)
    branch, bt = (4, 2, 2), 8
    nodes, layers, hkv, d, ctx = 28, 48, 8, 256, 1216
    pages = -(-ctx // 16)
    hist = torch.randint(0, VG, (bt, ctx), generator=gen, device=device, dtype=torch.int32)
    n = torch.full((bt,), 1024, **i32)
    d0t, d0p = torch.zeros((2 * bt,), **i32), torch.zeros((2 * bt,), **i32)
    vt, vp, vs = (torch.zeros((bt * (nodes + 1),), **i32) for _ in range(3))
    vm = torch.zeros((bt * (nodes + 1),), dtype=torch.int64, device=device)
    tb = torch.zeros((bt,), **i32)
    record("tree_prepare", timed(lambda i: kernels.tree_prepare(hist, n, branch, ctx, d0t, d0p, vt, vp, vs, vm, tb), 1),
           0, 1, "tree_prepare_kernel: rows, positions, slots and ancestor masks of 8 trees (launch-bound)")
    am = torch.randint(0, 4, (bt * (nodes + 1),), generator=gen, device=device, dtype=torch.int32)
    vt.copy_(torch.randint(0, 4, (bt * (nodes + 1),), generator=gen, device=device, dtype=torch.int32))
    ot, oc, acc = torch.zeros((bt, 4), **i32), torch.zeros((bt,), **i32), torch.zeros((bt * 3,), **i32)
    record("tree_accept", timed(lambda i: kernels.tree_accept(am, vt, bt, branch, ot, oc, acc), 1), 0, 1,
           "tree_accept_kernel: the walk down 8 trees (launch-bound)")
    kc = torch.zeros((layers, bt * pages, hkv, 16, d), dtype=bf, device=device)
    vc = torch.zeros_like(kc)
    table = torch.arange(bt * pages, **i32).view(bt, pages)
    tb.fill_(1024)
    acc.copy_(torch.tensor([0, 4, 12] * bt, dtype=torch.int32))
    moved = bt * 3 * layers * hkv * d * 2 * 2 * 2  # 3 accepted nodes: read + write K and V
    record("tree_compact", timed(lambda i: kernels.tree_compact(kc, vc, table, tb, acc, 3, 3, bt), 1), moved, 1,
           "tree_compact_kernel: 3 accepted nodes x 48 layers of K/V moved per tree, 8 trees (Gemma-3-12B)")
    if rank == 0:
        total_us = sum(v["us_per_call"] for v in out.values())
        line = {"metric": "small-kernel times (acceptance, sampling, top-k, tree bookkeeping, embedding)",
                "value": round(total_us, 3), "unit": "us (sum over the kernels, one call each)", "n_gpus": world,
                "steps": args.steps, "warmup": 3, "ms_per_step": round(total_us / 1000, 5), "higher_is_better": False,
                "scaling": "weak", "vs_baseline": None, "dtype": "bf16 logits, int32 ids", "data": "synthetic",
                "config": {"workload": "small kernels at the configurations' shapes", "kernels": out,
                           "l2": "inputs rotate over copies larger than the 126 MB L2 where the data is that large"},
                "peak_source": pk["source"]}
        print(json.dumps(line), flush=True)


def run_verify_step(args, world: int, rank: int, local: int) -> None:
    """one verify step's qGEMM (K=3840, N=15360, M=5, W ~ N(0, 0.02)) and greedy acceptance
    of 4 drafts against a 151936-vocab logit row per verified row (logits = the projection's output tiled to
    151936 entries plus fixed noise), with 8 rotating weight copies (266 MB) so the weights cannot sit in L2."""
    import torch

    from ironmule_b200 import kernels

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    pk = peaks()
    gen = torch.Generator(device=device).manual_seed(0)
    copies = [kernels.Packed(*kernels.quantize((torch.randn((15360, 3840), generator=gen, device=device) * 0.02)
                                               .to(torch.bfloat16))) for _ in range(8)]
    m = args.rows or 5
    x = torch.randn((m, 3840), generator=gen, device=device).to(torch.bfloat16)
    y = torch.empty((m, 15360), dtype=torch.bfloat16, device=device)
    reps = -(-151936 // 15360)
    noise = (torch.randn((5, reps * 15360), generator=gen, device=device) * 1e-3).to(torch.bfloat16)
    logits = torch.empty((5, 151936), dtype=torch.bfloat16, device=device)
    drafts = torch.randint(0, 151936, (1, 4), generator=gen, device=device, dtype=torch.int32)
    ws = kernels.workspace(kernels.qgemm_packed_workspace_bytes(m, 15360, 3840), device)
    tokens = torch.empty((1, 5), dtype=torch.int32, device=device)
    count = torch.empty((1,), dtype=torch.int32, device=device)
    stream = torch.cuda.current_stream(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def gemms(n):
        for i in range(n):
            kernels.qgemm_packed(x, copies[i % 8], out=y, ws=ws)

    gemms(3)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        gemms(64)
    g.replay()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(5):
        g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    sec = e0.elapsed_time(e1) / 1000 / (5 * 64)
    algo = 15360 * 3840 * 9 // 16 + m * 3840 * 2 + m * 15360 * 2
    achieved = algo / sec / 1e9
    tflops = 2.0 * 15360 * 3840 * m / sec / 1e12
    workload = "BASELINE config 1 qGEMM" if m == 5 else f"config 1 qGEMM shape at {m} rows"
    line = {"metric": f"qGEMM HBM GB/s (verify step, K=3840, N=15360, M={m})", "value": round(achieved, 1),
            "unit": "GB/s", "n_gpus": world, "steps": 5 * 64, "warmup": 3, "ms_per_step": round(sec * 1e3, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16/4-bit",
            "data": "synthetic", "config": {"workload": workload, "rotating_weight_copies": 8,
                                            "qgemm_path": args.qgemm_path, "tflops": round(tflops, 2)},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": round(achieved / pk["hbm_gbs"], 4), "traffic": None}}
    if m > 32:  # many rows: the tensor pipe is the bound that matters
        line["roofline"] = {"bound": "tensor", "achieved": round(tflops, 2), "peak": pk["bf16_tflops"],
                            "unit": "TFLOP/s", "frac": round(tflops / pk["bf16_tflops"], 4), "traffic": None}
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_attention(args, world: int, rank: int, local: int) -> None:
    """One attention launch of a round, alone, through the fused entry point (q/k RMSNorm + RoPE + KV write +
    attention), 16-token pages, 4 rotating KV layer caches. --attn-case config3-verify: 32 sequences with lengths
    U[128, 2048] (seed 0), Qwen3-4B heads (32 q / 8 kv, head_dim 128), `--rows` (default 5) rows per sequence;
    config3-draft: the same sequences, Qwen3-0.6B heads (16 / 8), 1 row; config2-draft: 1 sequence of 520 keys,
    Qwen3-0.6B heads, 1 row. Bytes per launch: every visible key's K and V once (2 x 8 heads x 128 x 2 B per key)
    plus the qkv rows in and the output rows out."""
    import torch

    from ironmule_b200 import kernels

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    pk = peaks()
    gen = torch.Generator(device=device).manual_seed(0)
    case = args.attn_case
    b = 1 if case == "config2-draft" else 32
    hq, hkv, d = (32 if case == "config3-verify" else 16), 8, 128
    rows = (args.rows or 5) if case == "config3-verify" else 1
    lens = [520] if b == 1 else torch.randint(128, 2049, (b,), generator=torch.Generator().manual_seed(0)).tolist()
    cap = 2048 + 64
    pages = cap // 16
    copies = 4
    kc = [torch.randn((b * pages, hkv, 16, d), generator=gen, device=device).to(torch.bfloat16) for _ in range(copies)]
    vc = [torch.randn((b * pages, hkv, 16, d), generator=gen, device=device).to(torch.bfloat16) for _ in range(copies)]
    table = torch.arange(b * pages, dtype=torch.int32, device=device).reshape(b, pages)
    m = b * rows
    qkv = torch.randn((m, (hq + 2 * hkv) * d), generator=gen, device=device).to(torch.bfloat16)
    qn = torch.ones(d, dtype=torch.bfloat16, device=device)
    inv_freq = (1e6 ** (-2.0 * torch.arange(d // 2, device=device, dtype=torch.float32) / d)).contiguous()
    slots = torch.tensor([n - rows + i for n in lens for i in range(rows)], dtype=torch.int32, device=device)
    seq_rows = torch.arange(0, m + 1, rows, dtype=torch.int32, device=device)
    out = torch.empty((m, hq * d), dtype=torch.bfloat16, device=device)
    ws = kernels.workspace(kernels.attention_workspace_bytes(b, rows, hq, hkv, d, cap, args.kpc), device)
    stream = torch.cuda.current_stream(device)

    def launches(n):
        for i in range(n):
            kernels.attention_qkv(qkv, qn, qn, inv_freq, slots, kc[i % copies], vc[i % copies], table, seq_rows, slots,
                                  hq=hq, hkv=hkv, d=d, eps=1e-6, max_rows_per_seq=rows, max_kv_len=cap,
                                  scale=d ** -0.5, keys_per_split=args.kpc, out=out, ws=ws)

    launches(max(args.warmup, 3))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        launches(32)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = max(1, args.steps // 32)
    e0.record(stream)
    for _ in range(reps):
        g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    sec = e0.elapsed_time(e1) / 1000 / (reps * 32)
    algo = sum(lens) * 2 * hkv * d * 2 + m * (hq + 2 * hkv) * d * 2 + m * hq * d * 2
    achieved = algo / sec / 1e9
    line = {"metric": f"attention HBM GB/s ({case}: {b} sequences, {hq}/{hkv} heads, {rows} rows each)",
            "value": round(achieved, 1), "unit": "GB/s", "n_gpus": world, "steps": reps * 32, "warmup": 3,
            "ms_per_step": round(sec * 1e3, 5), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"{case} attention, fused q/k norm + RoPE + KV write",
                       "kv_copies_rotating": copies, "bytes_per_launch": algo, "keys_per_split": args.kpc},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": round(achieved / pk["hbm_gbs"], 4), "traffic": None}}
    if rank == 0:
        print(json.dumps(line), flush=True)


# Qwen3-4B's projections as a GGUF file stores them (q, k, v apart): (N rows, K inputs)
KQ_SHAPES = ((4096, 2560), (1024, 2560), (1024, 2560), (2560, 4096), (9728, 2560), (9728, 2560), (2560, 9728))


def run_kquant(args, world: int, rank: int, local: int) -> None:
    """The ggml path's matmuls: every Q4_K projection of one Qwen3-4B token step (36 layers x 7, as the reference
    measures its generated kernels, ironmule/kernel_gen.py:16) at `--rows` tokens (default 1) through im_kq_gemv,
    captured as one CUDA graph; 2.04 GB of random Q4_K blocks (d, dmin ~ 2e-3), so no L2 flush is needed. Bytes per
    step: the weights once plus the float32 activations in and outputs out. cpu_baseline: the oracle's C product
    (one thread) over one layer's seven matrices."""
    import numpy as np
    import torch

    from ironmule_b200 import kernels
    from oracle import kquant as kq

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    pk = peaks()
    b = args.rows or 1
    layers = args.layers or 36
    gen = torch.Generator(device=device).manual_seed(0)
    weights, inputs, outputs = [], {}, []
    d = torch.tensor([2e-3, 2e-3], dtype=torch.float16).view(torch.uint8).to(device)
    for _ in range(layers):
        for n, k in KQ_SHAPES:
            w = torch.randint(0, 256, (n * (k // 256), 144), generator=gen, device=device, dtype=torch.uint8)
            w[:, 0:4] = d
            weights.append((w.reshape(-1), n, k))
            outputs.append(torch.empty((b, n), dtype=torch.float32, device=device))
    for n, k in KQ_SHAPES:
        inputs.setdefault(k, torch.randn((b, k), generator=gen, device=device))
    ws = kernels.workspace(max(kernels.kq_workspace_bytes(k, b) for _, k in KQ_SHAPES), device)
    stream = torch.cuda.current_stream(device)

    def step():
        for (w, n, k), y in zip(weights, outputs):
            kernels.kq_gemv(kernels.Q4_K, w, inputs[k], n, out=y, ws=ws)

    for _ in range(max(args.warmup, 3)):
        step()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    g.replay()
    torch.cuda.synchronize()
    clocks = Clocks(local)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    sec = e0.elapsed_time(e1) / 1000 / args.steps
    wbytes = sum(w.numel() for w, _, _ in weights)
    algo = wbytes + layers * sum(4 * b * (n + k) for n, k in KQ_SHAPES)
    achieved = algo / sec / 1e9
    # the CPU port: one layer's seven matrices at b tokens, one thread
    host = [(w.cpu().numpy(), n, k) for w, n, k in weights[:len(KQ_SHAPES)]]
    xs = {k: v.cpu().numpy() for k, v in inputs.items()}
    t0 = time.perf_counter()
    for w, n, k in host:
        kq.gemv(kq.Q4_K, w, n, xs[k])
    cpu_sec = time.perf_counter() - t0
    cpu_gbs = sum(w.size for w, _, _ in host) / cpu_sec / 1e9
    line = {"metric": f"Q4_K matmul GB/s (all Q4_K matmuls of a Qwen3-4B token step, {b} token(s))",
            "value": round(achieved, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": round(sec * 1e3, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8 x 4/6-bit integer dot, fp32 scales",
            "data": "synthetic (random Q4_K blocks, normal activations)",
            "config": {"workload": f"GGUF Q4_K matmuls of one Qwen3-4B token step ({layers} x 7 projections)",
                       "tokens": b, "weight_bytes": wbytes, "l2": f"{wbytes / 1e9:.2f} GB of weights per step > "
                                                                    "126 MB L2"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": round(achieved / pk["hbm_gbs"], 4), "traffic": None,
                         "kernel": f"kq_q4k_kernel + kq_quant_kernel, {len(weights)} pairs per step"},
            "cpu_baseline": {"value": round(cpu_gbs, 3), "unit": "GB/s", "cores": 1, "kind": "port",
                             "sample": f"one layer's 7 Q4_K matrices at {b} token(s), oracle/kquant_oracle.c"},
            "gpu_launches": 2 * len(weights) * args.steps, "clocks": clk, "peak_source": pk["source"]}
    if rank == 0:
        print(json.dumps(line), flush=True)


TP_SEQS, TP_PROMPT, TP_CTX = 64, 512, 512 + 256


def tp_decoder(device, world: int, rank: int, group):
    """BASELINE config 5a: Gemma-3-27B shapes tensor-parallel over the `world` ranks of `group` (NCCL all-reduce
    after o and down, the vocabulary-sharded head all-gathered), a replicated Gemma-3-1B-shaped draft, greedy,
    k = 4, 64 sequences of 512-token prompts (the same sequences on every rank: one job)."""
    import torch

    from ironmule_b200.engine import PRESETS, QuantModel, SpecDecoder

    b = TP_SEQS
    gen = torch.Generator().manual_seed(0)
    target = QuantModel(PRESETS["gemma3-27b"], device, seed=0, max_ctx=TP_CTX, max_seqs=b, max_rows=b * (K_DRAFTS + 1),
                        max_logit_rows=b * (K_DRAFTS + 1), tp=world, rank=rank, group=group)
    draft = QuantModel(PRESETS["gemma3-1b"], device, seed=1, max_ctx=TP_CTX, max_seqs=b, max_rows=2 * b,
                       max_logit_rows=2 * b)
    dec = SpecDecoder(target, draft, k=K_DRAFTS, batch=b)
    prompts = [torch.randint(0, target.cfg.vocab, (TP_PROMPT,), generator=gen, dtype=torch.int32) for _ in range(b)]
    return target, draft, dec, prompts


def tp_record(world: int, rank: int, local: int, steps: int = 5, warmup: int = 2) -> dict:
    """Config 5a at TP = world beside the replicas line: tokens/s and ms per round from graph-replayed rounds (CUDA
    events, max over ranks), and the collectives' share of a round, from one eager round with CUDA events around
    each NCCL call (all-reduces after o and down, the head's all-gather), against that eager round's time."""
    import gc

    import torch

    device = torch.device("cuda", local)
    group = None
    if world > 1:
        import torch.distributed as dist
        group = dist.group.WORLD
    target, draft, dec, prompts = tp_decoder(device, world, rank, group)
    try:
        dec.start([p.to(device) for p in prompts], max_new=TP_CTX - TP_PROMPT - dec.reserve - 8)
        dec.round()
        torch.cuda.synchronize()
        dec.capture()
        dec.run_rounds(warmup)
        torch.cuda.synchronize()
        before = dec.read_stats()
        barrier(world)
        stream = torch.cuda.current_stream(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        dec.run_rounds(steps)
        e1.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        ms = reduce_max(e0.elapsed_time(e1), world) / steps
        tokens = dec.read_stats().tokens - before.tokens
        dec.graph = None  # a graph holding NCCL calls goes before anything else touches the group
        target.collective_events = []
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        dec.round()
        g1.record(stream)
        torch.cuda.synchronize()
        coll_ms = sum(a.elapsed_time(b) for a, b in target.collective_events)
        calls = len(target.collective_events)
        eager_ms = g0.elapsed_time(g1)
        target.collective_events = None
        coll_ms, eager_ms = reduce_max(coll_ms, world), reduce_max(eager_ms, world)
        return {"workload": "config 5a: Gemma-3-27B shapes (4-bit) tensor-parallel, Gemma-3-1B-shaped draft replicated, "
                            f"greedy, k=4, {TP_SEQS} sequences, {TP_PROMPT}-token prompts",
                "tp": world, "value": round(tokens / (ms * steps / 1000), 2), "unit": "tokens/s",
                "ms_per_round": round(ms, 3), "steps": steps, "warmup": warmup, "scaling": "strong",
                "accepted_per_round": round((dec.read_stats().accepted - before.accepted) / steps, 3),
                "collectives_per_round": calls, "collective_ms_eager_round": round(coll_ms, 3),
                "eager_round_ms": round(eager_ms, 3),
                "collective_share": round(coll_ms / eager_ms, 4) if eager_ms > 0 else None}
    finally:
        dec.graph = None
        del dec, target, draft
        gc.collect()
        torch.cuda.empty_cache()


def run_rounds_workload(args, world: int, rank: int, local: int, kind: str) -> None:
    """Config 3 (stochastic, batched) or config 4 (tree) rounds: timed like the default workload."""
    import torch

    from ironmule_b200.engine import PRESETS, QuantModel, Sampling, SpecDecoder, TreeDecoder

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    pk = peaks()
    gen = torch.Generator().manual_seed(rank)
    tp_group = None
    if kind == "tp" and world > 1:
        import torch.distributed as dist
        tp_group = dist.group.WORLD
    if kind == "tp":
        ctx = TP_CTX
        target, draft, dec, prompts = tp_decoder(device, world, rank, tp_group)
        round_bytes = K_DRAFTS * draft.cfg.weight_bytes() + target.cfg.weight_bytes() // world
        workload = (f"BASELINE config 5a: Gemma-3-27B shapes (4-bit) tensor-parallel over {world} GPU(s), NCCL "
                    "all-reduce after o and down, vocabulary-sharded head all-gathered; replicated Gemma-3-1B-shaped "
                    "draft; greedy, k 4, 64 sequences (320 verify rows per qGEMM call), 512-token prompts")
        metric = "accepted tokens/s (spec decode, Gemma-3-27B tensor-parallel + 1B draft, k=4, 64 sequences)"
    elif kind == "stochastic":
        b, ctx = 32, 2048 + 256
        lens = torch.randint(128, 2049, (b,), generator=gen).tolist()
        target = QuantModel(PRESETS["qwen3-4b"], device, seed=0, max_ctx=ctx, max_seqs=b, max_rows=b * (K_DRAFTS + 1),
                            max_logit_rows=b * (K_DRAFTS + 1))
        draft = QuantModel(PRESETS["qwen3-0.6b"], device, seed=1, max_ctx=ctx, max_seqs=b, max_rows=2 * b,
                           max_logit_rows=2 * b)
        dec = SpecDecoder(target, draft, k=K_DRAFTS, batch=b, sampling=Sampling(0.7, 0.95, 0))
        prompts = [torch.randint(0, target.cfg.vocab, (n,), generator=gen, dtype=torch.int32) for n in lens]
        round_bytes = K_DRAFTS * draft.cfg.weight_bytes() + target.cfg.weight_bytes()
        workload = ("BASELINE config 3: stochastic speculative decoding (T 0.7, top-p 0.95, k 4, rejection sampling "
                    "with residual resample on Philox), Qwen3-4B + Qwen3-0.6B 4-bit, 32 concurrent sequences (160 "
                    "verify rows per qGEMM call), paged KV with 16-token pages, prompts U[128, 2048]")
        metric = "accepted tokens/s (stochastic spec decode, Qwen3-4B + 0.6B, k=4, 32 sequences)"
    else:
        b, ctx = 8, 1024 + 128 + 64
        target = QuantModel(PRESETS["gemma3-12b"], device, seed=0, max_ctx=ctx, max_seqs=b, max_rows=29 * b,
                            max_logit_rows=29 * b)
        draft = QuantModel(PRESETS["gemma3-1b"], device, seed=1, max_ctx=ctx, max_seqs=b, max_rows=8 * b,
                           max_logit_rows=8 * b)
        dec = TreeDecoder(target, draft, branch=(4, 2, 2), batch=b)
        prompts = [torch.randint(0, target.cfg.vocab, (1024,), generator=gen, dtype=torch.int32) for _ in range(b)]
        round_bytes = 3 * draft.cfg.weight_bytes() + target.cfg.weight_bytes()
        workload = ("BASELINE config 4: greedy tree verification, Gemma-3-12B shapes (4-bit) with a Gemma-3-1B-shaped "
                    "draft, 4 x 2 x 2 draft tree verified as root + 28 nodes (29 rows) per sequence, 8 sequences "
                    "(232 verify rows per qGEMM call), 1024-token prompts")
        metric = "accepted tokens/s (tree spec decode, Gemma-3-12B + 1B draft, 4x2x2 tree, 8 sequences)"
    room = max(8, ctx - max(p.numel() for p in prompts) - dec.reserve - 8)
    dev_prompts = [p.to(device) for p in prompts]
    torch.cuda.synchronize()
    t_prefill = time.perf_counter()
    dec.start(dev_prompts, max_new=room)  # both models' prefill, sequences packed into many-row forwards
    torch.cuda.synchronize()
    prefill_ms = (time.perf_counter() - t_prefill) * 1000
    dec.round()
    torch.cuda.synchronize()
    dec.capture()
    clocks = Clocks(local)
    clocks.start()
    dec.run_rounds(args.warmup)
    torch.cuda.synchronize()
    before = dec.read_stats()
    stream = torch.cuda.current_stream(device)
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    torch.cuda.nvtx.range_push("timed_rounds")
    dec.run_rounds(args.steps)
    torch.cuda.nvtx.range_pop()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    after = dec.read_stats()
    tokens = after.tokens - before.tokens
    max_ms = reduce_max(ms, world)
    # replicas add their sequences; a tensor-parallel job's ranks share the same ones
    total = float(tokens) if kind == "tp" else reduce_sum(float(tokens), world)
    value = total / (max_ms / 1000)
    step_s = max_ms / args.steps / 1000
    dec.graph = None  # a graph holding NCCL calls goes before the process group
    if rank == 0:
        line = {"metric": metric, "value": round(value, 3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(max_ms / args.steps, 4), "higher_is_better": True,
                "scaling": "strong" if kind == "tp" else "weak", "vs_baseline": None,
                "dtype": "bf16 activations, 4-bit weights (MLX affine g64)",
                "data": "synthetic (random-init weights, uniform random prompts)",
                "config": {"workload": workload,
                           "parallelism": f"tp{world}" if kind == "tp" else f"replicas x{world}",
                           "accepted_per_round": round((after.accepted - before.accepted) / args.steps, 4),
                           "round_weight_bytes": round_bytes,
                           "prefill_ms": round(prefill_ms, 1),
                           "prefill_tokens": sum(p.numel() - 1 for p in prompts)},
                "roofline": {"bound": "hbm", "achieved": round(round_bytes / step_s / 1e9, 1), "peak": pk["hbm_gbs"],
                             "unit": "GB/s", "frac": round(round_bytes / step_s / 1e9 / pk["hbm_gbs"], 4),
                             "traffic": None, "kernel": "whole round (weights streamed per round / round time)"},
                "clocks": clk, "gpu_launches": dec.launches_per_round() * args.steps, "peak_source": pk["source"]}
        print(json.dumps(line), flush=True)


def main() -> int:
    args = parse()
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, int(os.environ.get("WORLD_SIZE", "1")), rank)
        return 0
    world, rank, local = dist_setup(args)
    if args.qgemm_path:
        from ironmule_b200 import kernels
        kernels.qgemm_packed_path(args.qgemm_path)
    try:
        if args.workload == "verify_step":
            run_verify_step(args, world, rank, local)
        elif args.workload == "qgemm_pass":
            run_qgemm_pass(args, world, rank, local)
        elif args.workload == "small_kernels":
            run_small_kernels(args, world, rank, local)
        elif args.workload == "prefill":
            run_prefill(args, world, rank, local)
        elif args.workload == "attention":
            run_attention(args, world, rank, local)
        elif args.workload == "kquant":
            run_kquant(args, world, rank, local)
        elif args.workload in ("stochastic", "tree", "tp"):
            run_rounds_workload(args, world, rank, local, args.workload)
        else:
            run_spec_decode(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
