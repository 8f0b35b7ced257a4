"""TEST INFRASTRUCTURE ONLY -- the CPU oracle for the speculative-decoding hot path.

Only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s `cpu_baseline` / `--impl reference` arm may
import anything from this package, and only as the checker or the timed CPU baseline. The product
(`ironmule_b200`) never imports it and has no CPU fallback.

Contents:
  bf16.py       bfloat16 <-> float32 bit conversions (round to nearest even).
  quant.py      MLX-affine 4-bit group-64 quantiser / dequantiser (numpy).
  qmv.py        ctypes wrapper of qmv_oracle.c, the reference's qmv arithmetic in C.
  philox.py     Philox4x32-10 counter RNG (Salmon et al., SC'11).
  accept.py     greedy acceptance (IronMule ironmule/speculation.py:103-108), vocab argmax and top-1
                probability (ironmule/ggml_engine.py:669-683), stochastic acceptance (published
                speculative-sampling rule; no reference code exists).
  attention.py  paged verification attention with causal / tree masks.
  model.py      Qwen3 / Gemma-3 shaped forward passes on 4-bit weights.
"""
