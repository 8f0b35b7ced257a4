"""Makes the GGUF k-quant fixtures with the `gguf` package (gguf-py 0.19.0, ggml's own Python implementation of the
file format and of the Q4_K / Q6_K block decoding), run once in a container that has it:

    python tests/golden/make_kquant_golden.py

- kquant_golden.npz: seeded random Q4_K and Q6_K blocks and their float32 values from gguf.quants.dequantize;
- tiny.gguf: a small GGUF file written by gguf.GGUFWriter (metadata of several types; Q4_K, Q6_K, F32 and F16
  tensors);
- tiny_gguf.json: what gguf.GGUFReader reports for it (metadata values; per tensor its type, dimensions, byte count
  and the SHA-256 of its data).
The tests read these files only; they never import gguf.
"""
from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

import gguf  # noqa: E402

from oracle import kquant  # noqa: E402


def main() -> None:
    q4 = kquant.random_blocks(kquant.Q4_K, 24, seed=101)
    q6 = kquant.random_blocks(kquant.Q6_K, 24, seed=202)
    np.savez_compressed(
        HERE / "kquant_golden.npz", q4k_blocks=q4, q6k_blocks=q6,
        q4k_values=gguf.quants.dequantize(q4.reshape(-1), gguf.GGMLQuantizationType.Q4_K).astype(np.float32),
        q6k_values=gguf.quants.dequantize(q6.reshape(-1), gguf.GGMLQuantizationType.Q6_K).astype(np.float32))

    path = HERE / "tiny.gguf"
    w = gguf.GGUFWriter(str(path), arch="qwen3")
    w.add_uint32("qwen3.block_count", 1)
    w.add_uint32("qwen3.embedding_length", 512)
    w.add_float32("qwen3.rope.freq_base", 1000000.0)
    w.add_bool("tokenizer.ggml.add_bos_token", False)
    w.add_string("general.name", "tiny k-quant fixture")
    w.add_array("tokenizer.ggml.tokens", ["<a>", "<b>", "c"])
    w.add_array("qwen3.some_ints", [3, 1, 4])
    w.add_tensor("blk.0.ffn_down.weight", kquant.random_blocks(kquant.Q4_K, 4 * 2, seed=7).reshape(4, 2 * 144),
                 raw_dtype=gguf.GGMLQuantizationType.Q4_K)
    w.add_tensor("output.weight", kquant.random_blocks(kquant.Q6_K, 3, seed=8).reshape(3, 210),
                 raw_dtype=gguf.GGMLQuantizationType.Q6_K)
    w.add_tensor("output_norm.weight", np.linspace(-1, 1, 512, dtype=np.float32))
    w.add_tensor("token_embd.weight", np.arange(6, dtype=np.float16).reshape(2, 3))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()

    r = gguf.GGUFReader(str(path))
    meta = {}
    for field in r.fields.values():
        if field.name.startswith("GGUF."):
            continue
        meta[field.name] = field.contents()
    tensors = {}
    for t in r.tensors:
        data = np.asarray(t.data).tobytes()
        tensors[t.name] = {"type": int(t.tensor_type), "dims": [int(v) for v in t.shape],
                           "n_bytes": int(t.n_bytes), "offset": int(t.data_offset),
                           "sha256": hashlib.sha256(data).hexdigest()}
    (HERE / "tiny_gguf.json").write_text(json.dumps({"metadata": meta, "tensors": tensors,
                                                    "alignment": int(r.alignment)}, indent=1) + "\n")


if __name__ == "__main__":
    main()
