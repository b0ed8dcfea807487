"""Generate the committed golden fixtures for the Q4_K path.

Run from the repository root:  python tests/golden/make_golden.py

The reference (TypeScript + WGSL) cannot run in this container and ships no
fixtures for this path, so the fixtures come from independent
implementations of the algorithms it cites:

* q4k_blocks.npz -- Q4_K super-blocks (seeded random plus hand-built edge
  cases) decoded by the `gguf` Python package 0.19.0 (gguf-py's
  Q4_K.dequantize_blocks, the published llama.cpp dequantize_row_q4_K that
  src/gguf.ts:164-166 names as its layout source), and the f16 bit patterns
  numpy's IEEE round-to-nearest-even cast gives for those values (what
  Float16Array.set does at src/gguf.ts:432-436).
* gemv_c0.npz -- config 0 (2048 x 1536, M=1): y computed in float64 from the
  gguf-py weights rounded to f16, plus a digest of the synthetic bytes so a
  generator change is caught.
* q6k_blocks.npz -- Q6_K super-blocks (seeded random plus hand-built edge
  cases: extreme int8 scales, every 6-bit quant, subnormal / huge / NaN d)
  decoded by gguf-py's Q6_K.dequantize_blocks (llama.cpp's
  dequantize_row_q6_K, the layout src/gguf.ts:316-368 decodes) and the RNE
  f16 bit patterns of those values.
* q5k_blocks.npz -- Q5_K super-blocks (seeded random plus hand-built edge
  cases: every 5-bit quant with each qh bit, max scales/mins, subnormal and
  NaN d, negative dmin) decoded by gguf-py's Q5_K.dequantize_blocks
  (llama.cpp's dequantize_row_q5_K, the layout src/gguf.ts:212-314 decodes)
  and the RNE f16 bit patterns of those values (what the per-layer embedding
  upload stores, src/engine.ts:697-702).
* select.npz -- small logit vectors with planted ties, NaN and -1e30 entries,
  with argmax / per-residue max computed by a numpy restatement of
  shaders/argmax.wgsl and shaders/topk256.wgsl.
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "gemma4-webgpu_b200"))

from q4k import synth  # noqa: E402

OUT = Path(__file__).resolve().parent


def gguf_dequant(blocks: np.ndarray) -> np.ndarray:
    from gguf import quants
    from gguf.constants import GGMLQuantizationType

    with np.errstate(all="ignore"):
        return quants.dequantize(blocks.reshape(-1), GGMLQuantizationType.Q4_K).astype(np.float32).reshape(-1)


def edge_blocks() -> np.ndarray:
    """Hand-built super-blocks for the cases the decode must get right."""
    blocks = []

    def blk(d, dmin, sc, mn, qs):
        b = np.zeros(144, dtype=np.uint8)
        b[0:2] = np.array([d], dtype=np.float16).view(np.uint8)
        b[2:4] = np.array([dmin], dtype=np.float16).view(np.uint8)
        b[4:16] = synth.pack_scale_min(np.array([sc]), np.array([mn]))[0]
        b[16:] = qs
        return b

    rng = np.random.Generator(np.random.PCG64(7))
    ramp = np.arange(128, dtype=np.uint8)  # nibbles 0..15 in both halves
    blocks.append(np.zeros(144, dtype=np.uint8))                                  # all zero
    blocks.append(blk(1.0, 0.0, [1] * 8, [0] * 8, ramp))                           # w = q
    blocks.append(blk(1.0, 1.0, list(range(8)), list(range(8, 16)), ramp))         # distinct (sc, m)
    for j in range(8):                                                             # one slot at 63
        sc = [0] * 8
        mn = [0] * 8
        sc[j] = 63
        mn[j] = 48
        blocks.append(blk(0.5, 0.25, sc, mn, ramp))
    blocks.append(blk(6.0e-8, 6.0e-8, [63] * 8, [63] * 8, ramp))                  # f16 subnormal d, dmin
    blocks.append(blk(1.0e-3, 3.0e-3, [63] * 8, [63] * 8, ramp))                  # results near zero
    blocks.append(blk(60000.0, 0.0, [63] * 8, [0] * 8, ramp))                      # overflows f16 -> inf
    blocks.append(blk(70.0, 1.0, [63] * 8, [63] * 8, ramp))                        # f16-normal large values
    blocks.append(blk(2.0 ** -14, 2.0 ** -15, [33] * 8, [17] * 8, ramp))           # RNE ties in the subnormal range
    blocks.append(blk(1.0 / 1024, 0.0, [3] * 8, [0] * 8, rng.integers(0, 256, 128, dtype=np.uint8)))
    b = blk(1.0, 0.0, [1] * 8, [0] * 8, ramp)                                      # NaN d
    b[0:2] = np.array([0x7E00], dtype=np.uint16).view(np.uint8)
    blocks.append(b)
    b = blk(1.0, 0.0, [0] * 8, [0] * 8, ramp)                                      # inf d, sc = 0 -> NaN
    b[0:2] = np.array([0x7C00], dtype=np.uint16).view(np.uint8)
    blocks.append(b)
    b = rng.integers(0, 256, 144, dtype=np.uint8)                                  # raw random bytes
    b[0:2] = np.array([0x1234], dtype=np.uint16).view(np.uint8)
    b[2:4] = np.array([0x0456], dtype=np.uint16).view(np.uint8)
    blocks.append(b)
    return np.stack(blocks)


def make_blocks_fixture() -> None:
    rng = np.random.Generator(np.random.PCG64(synth.seed_for(0, 999)))
    rand = synth.make_blocks(64, rng)
    wide = synth.make_blocks(32, np.random.Generator(np.random.PCG64(11)), d_sigma=0.5)
    blocks = np.concatenate([edge_blocks(), rand, wide]).astype(np.uint8)
    f32 = gguf_dequant(blocks)
    with np.errstate(all="ignore"):
        f16 = f32.astype(np.float16).view(np.uint16)
    np.savez_compressed(OUT / "q4k_blocks.npz", blocks=blocks, f32=f32, f16=f16)


def q6k_edge_blocks() -> np.ndarray:
    """Hand-built Q6_K super-blocks: ql | qh | int8 scales | f16 d."""
    def blk(d, scales, ql, qh):
        b = np.zeros(210, dtype=np.uint8)
        b[0:128] = ql
        b[128:192] = qh
        b[192:208] = np.array(scales, dtype=np.int8).view(np.uint8)
        b[208:210] = np.array([d], dtype=np.float16).view(np.uint8)
        return b

    rng = np.random.Generator(np.random.PCG64(17))
    ramp_ql = np.arange(128, dtype=np.uint8) * 3
    ramp_qh = np.arange(64, dtype=np.uint8) * 5
    out = [np.zeros(210, dtype=np.uint8)]
    out.append(blk(1.0, [1] * 16, ramp_ql, ramp_qh))                       # w = q - 32
    out.append(blk(1.0, [-128] * 16, np.full(128, 0xFF, np.uint8), np.full(64, 0xFF, np.uint8)))  # q = 31
    out.append(blk(1.0, [-128] * 16, np.zeros(128, np.uint8), np.zeros(64, np.uint8)))  # q = -32: 4096
    out.append(blk(1.0, [127] * 16, ramp_ql, ramp_qh))                     # |sc*q| > 2048, odd products
    out.append(blk(2.0 ** -10, list(range(-128, 128, 16)), ramp_ql, ramp_qh))
    out.append(blk(6.0e-8, [127, -128] * 8, ramp_ql, ramp_qh))            # subnormal d
    out.append(blk(3.0, [127] * 16, ramp_ql, ramp_qh))                     # results past f16 max -> inf
    out.append(blk(1.0e-3, [-77, 91, 33, -5, 101, -128, 127, 1] * 2, rng.integers(0, 256, 128, dtype=np.uint8),
                   rng.integers(0, 256, 64, dtype=np.uint8)))
    b = blk(1.0, [1] * 16, ramp_ql, ramp_qh)                               # NaN d
    b[208:210] = np.array([0x7E00], dtype=np.uint16).view(np.uint8)
    out.append(b)
    b = blk(1.0, [0] * 16, ramp_ql, ramp_qh)                               # inf d, sc = 0 -> NaN
    b[208:210] = np.array([0x7C00], dtype=np.uint16).view(np.uint8)
    out.append(b)
    return np.stack(out)


def make_q6k_fixture() -> None:
    from gguf import quants
    from gguf.constants import GGMLQuantizationType

    rand = synth.make_q6k_blocks(64, np.random.Generator(np.random.PCG64(synth.seed_for(0, 998))))
    wide = synth.make_q6k_blocks(32, np.random.Generator(np.random.PCG64(12)), d_sigma=0.05)
    blocks = np.concatenate([q6k_edge_blocks(), rand, wide]).astype(np.uint8)
    with np.errstate(all="ignore"):
        f32 = quants.dequantize(blocks.reshape(-1), GGMLQuantizationType.Q6_K).astype(np.float32).reshape(-1)
        f16 = f32.astype(np.float16).view(np.uint16)
    np.savez_compressed(OUT / "q6k_blocks.npz", blocks=blocks, f32=f32, f16=f16)


def q5k_edge_blocks() -> np.ndarray:
    """Hand-built Q5_K super-blocks: d | dmin | scales | qh | qs."""
    def blk(d, dmin, sc, mn, qh, qs):
        b = np.zeros(176, dtype=np.uint8)
        b[0:2] = np.array([d], dtype=np.float16).view(np.uint8)
        b[2:4] = np.array([dmin], dtype=np.float16).view(np.uint8)
        b[4:16] = synth.pack_scale_min(np.array([sc]), np.array([mn]))[0]
        b[16:48] = qh
        b[48:176] = qs
        return b

    ramp_qs = (np.arange(128) * 37 % 256).astype(np.uint8)
    ramp_qh = (np.arange(32) * 11 % 256).astype(np.uint8)
    out = [np.zeros(176, dtype=np.uint8)]
    out.append(blk(1.0, 0.0, [1] * 8, [0] * 8, np.zeros(32, np.uint8), ramp_qs))            # q without the 5th bit
    out.append(blk(1.0, 0.0, [1] * 8, [0] * 8, np.full(32, 0xFF, np.uint8), ramp_qs))      # q + 16
    out.append(blk(1.0, 1.0, [63] * 8, [63] * 8, np.full(32, 0xFF, np.uint8), np.full(128, 0xFF, np.uint8)))
    out.append(blk(0.5, 0.25, list(range(0, 64, 8)), list(range(63, -1, -8)), ramp_qh, ramp_qs))
    out.append(blk(6.0e-8, 6.0e-8, [63, 1] * 4, [1, 63] * 4, ramp_qh, ramp_qs))               # subnormal d, dmin
    out.append(blk(2.0e-3, -3.0e-3, [17, 42, 5, 63, 0, 31, 48, 9], [3, 60, 22, 0, 63, 7, 14, 40], ramp_qh, ramp_qs))
    out.append(blk(40.0, 0.0, [63] * 8, [0] * 8, np.full(32, 0xFF, np.uint8), np.full(128, 0xFF, np.uint8)))  # > f16 max
    b = blk(1.0, 1.0, [1] * 8, [1] * 8, ramp_qh, ramp_qs)                                    # NaN d
    b[0:2] = np.array([0x7E00], dtype=np.uint16).view(np.uint8)
    out.append(b)
    return np.stack(out)


def make_q5k_fixture() -> None:
    from gguf import quants
    from gguf.constants import GGMLQuantizationType

    rand = synth.make_q5k_blocks(64, np.random.Generator(np.random.PCG64(synth.seed_for(0, 997))))
    wide = synth.make_q5k_blocks(32, np.random.Generator(np.random.PCG64(13)), d_sigma=0.5)
    blocks = np.concatenate([q5k_edge_blocks(), rand, wide]).astype(np.uint8)
    with np.errstate(all="ignore"):
        f32 = quants.dequantize(blocks.reshape(-1), GGMLQuantizationType.Q5_K).astype(np.float32).reshape(-1)
        f16 = f32.astype(np.float16).view(np.uint16)
    np.savez_compressed(OUT / "q5k_blocks.npz", blocks=blocks, f32=f32, f16=f16)


def make_gemv_fixture() -> None:
    M, N = 2048, 1536
    w = synth.q4k_matrix(M, N, synth.seed_for(0, 0))
    x = synth.activations(1, N, synth.seed_for(0, 100))
    w16 = gguf_dequant(w).astype(np.float16).astype(np.float64).reshape(M, N)
    y = w16 @ x[0].astype(np.float64)
    np.savez_compressed(
        OUT / "gemv_c0.npz",
        y=y,
        w_sha256=np.frombuffer(hashlib.sha256(w.tobytes()).digest(), dtype=np.uint8),
        x_sha256=np.frombuffer(hashlib.sha256(x.tobytes()).digest(), dtype=np.uint8),
        M=M,
        N=N,
    )


def select_reference(v: np.ndarray):
    """numpy restatement of argmax.wgsl / topk256.wgsl (first strict max per
    residue from -1e30, tree keeps the lower lane on ties)."""
    n = v.size
    vals = np.full(256, -1e30, dtype=np.float32)
    idx = np.zeros(256, dtype=np.uint32)
    for t in range(256):
        for i in range(t, n, 256):
            if v[i] > vals[t]:
                vals[t] = v[i]
                idx[t] = i
    mx = vals.copy()
    ix = idx.copy()
    stride = 128
    while stride:
        for t in range(stride):
            if mx[t + stride] > mx[t]:
                mx[t] = mx[t + stride]
                ix[t] = ix[t + stride]
        stride >>= 1
    return int(ix[0]), vals, idx


def make_select_fixture() -> None:
    rng = np.random.Generator(np.random.PCG64(5))
    cases = {}
    v = rng.standard_normal(4096).astype(np.float32) * 10
    cases["plain"] = v
    t = v.copy()
    t[[700, 1212, 3000]] = 99.0            # global tie in different residues
    t[[17, 17 + 512, 17 + 1024]] = 50.0     # tie inside one residue
    cases["ties"] = t
    n = v.copy()
    n[::7] = np.nan                         # NaN never wins
    n[5] = -1e30
    cases["nan"] = n
    lo = np.full(1024, -1e30, dtype=np.float32)
    lo[[3, 300]] = -2e30                    # nothing beats the -1e30 start
    cases["floor"] = lo
    cases["ragged"] = rng.standard_normal(1000).astype(np.float32)   # n not a multiple of 256
    cases["tiny"] = rng.standard_normal(37).astype(np.float32)       # n < 256
    out = {}
    for k, arr in cases.items():
        am, vals, idx = select_reference(arr)
        out[f"{k}_logits"] = arr
        out[f"{k}_argmax"] = np.array(am, dtype=np.uint32)
        out[f"{k}_vals"] = vals
        out[f"{k}_idx"] = idx
    np.savez_compressed(OUT / "select.npz", **out)


if __name__ == "__main__":
    make_blocks_fixture()
    make_q6k_fixture()
    make_q5k_fixture()
    make_gemv_fixture()
    make_select_fixture()
    for f in sorted(OUT.glob("*.npz")):
        print(f.name, f.stat().st_size)
