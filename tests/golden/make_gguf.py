"""Generate tests/golden/tiny_q4k.gguf, the GGUF fixture of the reader tests.

Run from the repository root:  python tests/golden/make_gguf.py

The file is written by the `gguf` Python package 0.19.0 (gguf-py's
GGUFWriter, the published GGUF v3 writer), not by this repository's code, so
the reader (gemma4-webgpu_b200/q4k/gguf.py, which restates src/gguf.ts:11-101)
is checked against an independent producer.  Contents:

* metadata of every value type 0-12 (scalars, a string, arrays of strings and
  of integers), with Gemma-style keys next to plain test keys;
* Q4_K matrices shaped like the reference's weights, stored as GGUF stores
  them (dims [N, M], ne0 = N): a 2-D `blk.0.attn_q.weight` (256 x 512) and a
  tied `token_embd.weight` (1024 x 256, the LM head's rows);
* one tensor of each other type the reference's tensorByteSize knows (F32
  norm vector, F16, BF16, Q8_0, Q5_K, Q6_K), so the offsets after them are
  exercised.

Seeded: rerunning reproduces the file byte for byte.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "gemma4-webgpu_b200"))

from q4k import synth  # noqa: E402

OUT = Path(__file__).resolve().parent / "tiny_q4k.gguf"


def main() -> None:
    import gguf
    from gguf.constants import GGMLQuantizationType as T

    rng = np.random.Generator(np.random.PCG64(2024))
    w = gguf.GGUFWriter(str(OUT), "gemma4")
    w.add_uint32("gemma4.block_count", 1)
    w.add_uint32("gemma4.embedding_length", 256)
    w.add_float32("gemma4.final_logit_softcapping", 30.0)
    w.add_string("general.name", "tiny q4k fixture")
    w.add_bool("test.flag", True)
    w.add_uint8("test.u8", 200)
    w.add_int8("test.i8", -100)
    w.add_uint16("test.u16", 60000)
    w.add_int16("test.i16", -30000)
    w.add_int32("test.i32", -2_000_000_000)
    w.add_uint64("test.u64", 2 ** 40 + 3)
    w.add_int64("test.i64", -(2 ** 40) - 5)
    w.add_float64("test.f64", 0.1)
    w.add_array("test.tokens", ["<pad>", "<bos>", "héllo"])
    w.add_array("test.ints", [1, -2, 3])

    # Q4_K matrices: synth.q4k_matrix returns [rows, cols/256*144] bytes
    w.add_tensor("blk.0.attn_q.weight", synth.q4k_matrix(256, 512, seed=11), raw_dtype=T.Q4_K)
    w.add_tensor("blk.0.attn_norm.weight", rng.standard_normal(256).astype(np.float32))
    w.add_tensor("blk.0.f16.weight", rng.standard_normal((4, 64)).astype(np.float16))
    w.add_tensor("blk.0.bf16.weight", rng.integers(0, 2 ** 16, (2, 32), dtype=np.uint16).view(np.uint8)
                 .reshape(2, 64), raw_dtype=T.BF16)
    w.add_tensor("blk.0.q8_0.weight", rng.integers(0, 256, (3, 2 * 34), dtype=np.uint8), raw_dtype=T.Q8_0)
    w.add_tensor("blk.0.q5_k.weight", rng.integers(0, 256, (2, 176), dtype=np.uint8), raw_dtype=T.Q5_K)
    w.add_tensor("blk.0.q6_k.weight", rng.integers(0, 256, (3, 210), dtype=np.uint8), raw_dtype=T.Q6_K)
    w.add_tensor("token_embd.weight", synth.q4k_matrix(1024, 256, seed=12), raw_dtype=T.Q4_K)

    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
