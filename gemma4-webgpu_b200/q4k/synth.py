"""Seeded synthetic Q4_K weights and f32 activations.

The reference measures on a real Gemma-4-E2B Q4_K_M GGUF, which is not
available here; the benchmark configurations instead use seeded synthetic
super-blocks with the distribution below.  Every super-block follows the GGUF
Q4_K layout that src/gguf.ts:157-210 decodes:

    offset 0   f16 d        = f16(|N(0, 2e-3)|)
    offset 2   f16 dmin     = f16(|N(0, 2e-3)|)
    offset 4   12 bytes     8 (scale, min) pairs, 6 bits each, uniform in [0, 63] (low
                            6 bits of uniform random bytes),
                            packed as the exact inverse of getScaleMin
                            (src/gguf.ts:175-182)
    offset 16  128 bytes    256 nibbles, uniform in [0, 15]

Q6_K super-blocks (src/gguf.ts:316-368 layout, 210 bytes) for the Q6_K
GEMV: ql[128] and qh[64] uniform random bytes (6-bit quants uniform in
[0, 63]), 16 int8 scales uniform in [-128, 127], f16 d = f16(|N(0, 2e-5)|)
(weights of the same magnitude as the Q4_K ones).

Random numbers come from numpy Generator(PCG64(seed)) with
seed = 20261201 + 1000 * config + matrix_id.
"""
from __future__ import annotations

import numpy as np

QK_K = 256
BLOCK_BYTES = 144
SEED_BASE = 20261201


def seed_for(config: int, matrix_id: int) -> int:
    return SEED_BASE + 1000 * config + matrix_id


def pack_scale_min(sc: np.ndarray, mn: np.ndarray) -> np.ndarray:
    """Pack 8 six-bit scales and mins per block into the 12-byte field.

    Inverse of getScaleMin (src/gguf.ts:175-182): for j < 4 the low 6 bits of
    s[j] hold sc_j and of s[j+4] hold m_j; for j >= 4, s[j+4] holds the low
    nibbles of sc_j / m_j and the top two bits of s[j-4] / s[j] hold their high
    two bits.  sc, mn: uint8 [n_blocks, 8] in [0, 63].
    """
    sc = sc.astype(np.uint8)
    mn = mn.astype(np.uint8)
    out = np.empty((sc.shape[0], 12), dtype=np.uint8)
    out[:, 0:4] = sc[:, 0:4] | ((sc[:, 4:8] >> 4) << 6)
    out[:, 4:8] = mn[:, 0:4] | ((mn[:, 4:8] >> 4) << 6)
    out[:, 8:12] = (sc[:, 4:8] & 0x0F) | ((mn[:, 4:8] & 0x0F) << 4)
    return out


def unpack_scale_min(scales: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """getScaleMin over all 8 sub-blocks: [n, 12] bytes -> (sc, m) [n, 8]."""
    s = scales.astype(np.uint8)
    sc = np.empty((s.shape[0], 8), dtype=np.uint8)
    mn = np.empty_like(sc)
    sc[:, 0:4] = s[:, 0:4] & 0x3F
    mn[:, 0:4] = s[:, 4:8] & 0x3F
    sc[:, 4:8] = (s[:, 8:12] & 0x0F) | ((s[:, 0:4] >> 6) << 4)
    mn[:, 4:8] = (s[:, 8:12] >> 4) | ((s[:, 4:8] >> 6) << 4)
    return sc, mn


def make_blocks(n_blocks: int, rng: np.random.Generator, d_sigma: float = 2e-3) -> np.ndarray:
    """n_blocks seeded Q4_K super-blocks as uint8 [n_blocks, 144]."""
    d = np.abs(rng.normal(0.0, d_sigma, n_blocks)).astype(np.float16)
    dmin = np.abs(rng.normal(0.0, d_sigma, n_blocks)).astype(np.float16)
    # Uniform random bytes: the low 6 bits give uniform scales/mins in
    # [0, 63]; a whole byte gives two uniform nibbles in [0, 15].
    raw = np.frombuffer(rng.bytes(n_blocks * 144), dtype=np.uint8).reshape(n_blocks, 144)
    sc = raw[:, 0:8] & 0x3F
    mn = raw[:, 8:16] & 0x3F
    qs = raw[:, 16:144]
    out = np.empty((n_blocks, BLOCK_BYTES), dtype=np.uint8)
    out[:, 0:2] = d.view(np.uint8).reshape(n_blocks, 2)
    out[:, 2:4] = dmin.view(np.uint8).reshape(n_blocks, 2)
    out[:, 4:16] = pack_scale_min(sc, mn)
    out[:, 16:144] = qs
    return out


def q4k_matrix(rows: int, cols: int, seed: int) -> np.ndarray:
    """A [rows, cols] Q4_K weight as uint8 [rows, cols/256*144], row-major by
    super-block exactly as GGUF stores it (ne0 = cols is fastest)."""
    if cols % QK_K:
        raise ValueError(f"cols={cols} is not a multiple of {QK_K}")
    nb = cols // QK_K
    rng = np.random.Generator(np.random.PCG64(seed))
    return make_blocks(rows * nb, rng).reshape(rows, nb * BLOCK_BYTES)


def activations(batch: int, n: int, seed: int) -> np.ndarray:
    """f32 [batch, n] ~ N(0, 1)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    return rng.standard_normal((batch, n), dtype=np.float32)


def q4k_bytes(rows: int, cols: int) -> int:
    """Size rule of tensorByteSize for type 12 (src/gguf.ts:390)."""
    return rows * cols // QK_K * BLOCK_BYTES


Q6K_BLOCK_BYTES = 210


def make_q6k_blocks(n_blocks: int, rng: np.random.Generator, d_sigma: float = 2e-5) -> np.ndarray:
    """n_blocks seeded Q6_K super-blocks as uint8 [n_blocks, 210] (GGUF layout)."""
    out = np.frombuffer(rng.bytes(n_blocks * Q6K_BLOCK_BYTES), dtype=np.uint8).reshape(n_blocks, -1).copy()
    d = np.abs(rng.normal(0.0, d_sigma, n_blocks)).astype(np.float16)
    out[:, 208:210] = d.view(np.uint8).reshape(n_blocks, 2)
    return out


def q6k_matrix(rows: int, cols: int, seed: int) -> np.ndarray:
    """A [rows, cols] Q6_K weight as uint8 [rows, cols/256*210], GGUF row-major."""
    if cols % QK_K:
        raise ValueError(f"cols={cols} is not a multiple of {QK_K}")
    nb = cols // QK_K
    rng = np.random.Generator(np.random.PCG64(seed))
    return make_q6k_blocks(rows * nb, rng).reshape(rows, nb * Q6K_BLOCK_BYTES)


def q6k_bytes(rows: int, cols: int) -> int:
    """Size rule of tensorByteSize for type 14 (src/gguf.ts:392)."""
    return rows * cols // QK_K * Q6K_BLOCK_BYTES


Q5K_BLOCK_BYTES = 176


def make_q5k_blocks(n_blocks: int, rng: np.random.Generator, d_sigma: float = 2e-3) -> np.ndarray:
    """n_blocks seeded Q5_K super-blocks as uint8 [n_blocks, 176] (GGUF
    layout: f16 d, f16 dmin, 12 packed scale/min bytes, qh[32], qs[128]);
    d, dmin, scales and mins drawn as for Q4_K, qh and qs uniform bytes."""
    d = np.abs(rng.normal(0.0, d_sigma, n_blocks)).astype(np.float16)
    dmin = np.abs(rng.normal(0.0, d_sigma, n_blocks)).astype(np.float16)
    raw = np.frombuffer(rng.bytes(n_blocks * Q5K_BLOCK_BYTES), dtype=np.uint8).reshape(n_blocks, -1)
    out = np.empty((n_blocks, Q5K_BLOCK_BYTES), dtype=np.uint8)
    out[:, 0:2] = d.view(np.uint8).reshape(n_blocks, 2)
    out[:, 2:4] = dmin.view(np.uint8).reshape(n_blocks, 2)
    out[:, 4:16] = pack_scale_min(raw[:, 0:8] & 0x3F, raw[:, 8:16] & 0x3F)
    out[:, 16:176] = raw[:, 16:176]
    return out


def q5k_table(vocab: int, layers: int, seed: int) -> np.ndarray:
    """A per-layer embedding table [vocab, layers*256] in Q5_K as GGUF stores
    it: row v is `layers` consecutive super-blocks, block L = layer L's 256
    values (src/engine.ts:681-702)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    return make_q5k_blocks(vocab * layers, rng).reshape(vocab, layers * Q5K_BLOCK_BYTES)


def q5k_bytes(rows: int, cols: int) -> int:
    """Size rule of tensorByteSize for type 13 (src/gguf.ts:391)."""
    return rows * cols // QK_K * Q5K_BLOCK_BYTES
