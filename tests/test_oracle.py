"""CPU tests of the oracle: pinned against the golden fixtures (gguf-py Q4_K
decode, numpy RNE casts, numpy restatements of argmax/topk256) and
known-answer super-blocks built by hand from the layout of src/gguf.ts:157-210."""
from __future__ import annotations

import hashlib

import numpy as np
import pytest

from q4k import synth


def _f16_equal(a: np.ndarray, b: np.ndarray) -> bool:
    """Bit equality of f16 patterns, treating every NaN pattern as equal."""
    nan_a = ((a & 0x7C00) == 0x7C00) & ((a & 0x3FF) != 0)
    nan_b = ((b & 0x7C00) == 0x7C00) & ((b & 0x3FF) != 0)
    return np.array_equal(nan_a, nan_b) and np.array_equal(a[~nan_a], b[~nan_b])


def test_dequant_f32_matches_gguf_py(oracle, golden_dir):
    g = np.load(golden_dir / "q4k_blocks.npz")
    out = oracle.dequant_f32(g["blocks"])
    ref = g["f32"]
    assert np.array_equal(np.isnan(out), np.isnan(ref))
    m = ~np.isnan(ref)
    assert np.array_equal(out[m].view(np.uint32), ref[m].view(np.uint32))


def test_dequant_f16_matches_golden(oracle, golden_dir):
    g = np.load(golden_dir / "q4k_blocks.npz")
    assert _f16_equal(oracle.dequant_f16(g["blocks"]), g["f16"])


def test_truncating_fallback_differs(oracle, golden_dir):
    g = np.load(golden_dir / "q4k_blocks.npz")
    rne = oracle.dequant_f16(g["blocks"])
    tr = oracle.dequant_f16(g["blocks"], truncate=True)
    assert (rne != tr).sum() > 100  # the two f32ToF16Array paths are not interchangeable


def test_known_answer_identity_block(oracle):
    # d = 1, dmin = 0, every scale 1: each weight equals its nibble.
    b = np.zeros(144, dtype=np.uint8)
    b[0:2] = np.array([1.0], dtype=np.float16).view(np.uint8)
    b[4:16] = synth.pack_scale_min(np.ones((1, 8), np.uint8), np.zeros((1, 8), np.uint8))[0]
    b[16:] = np.arange(128, dtype=np.uint8)
    w = oracle.dequant_f32(b)
    qs = np.arange(128, dtype=np.uint8)
    for g in range(4):
        assert np.array_equal(w[64 * g: 64 * g + 32], (qs[32 * g: 32 * g + 32] & 15).astype(np.float32))
        assert np.array_equal(w[64 * g + 32: 64 * g + 64], (qs[32 * g: 32 * g + 32] >> 4).astype(np.float32))


@pytest.mark.parametrize("j", range(8))
def test_scale_min_slots(oracle, j):
    rng = np.random.default_rng(j)
    sc = rng.integers(0, 64, (1, 8), dtype=np.uint8)
    mn = rng.integers(0, 64, (1, 8), dtype=np.uint8)
    b = np.zeros(144, dtype=np.uint8)
    b[4:16] = synth.pack_scale_min(sc, mn)[0]
    assert oracle.scale_min(b, j) == (int(sc[0, j]), int(mn[0, j]))
    usc, umn = synth.unpack_scale_min(b[None, 4:16])
    assert usc[0, j] == sc[0, j] and umn[0, j] == mn[0, j]


def test_scale_min_high_bits(oracle):
    # j >= 4 reads its top two bits from s[j-4] / s[j] (src/gguf.ts:179-180).
    sc = np.array([[0, 0, 0, 0, 63, 48, 32, 16]], dtype=np.uint8)
    mn = np.array([[0, 0, 0, 0, 16, 32, 48, 63]], dtype=np.uint8)
    b = np.zeros(144, dtype=np.uint8)
    b[4:16] = synth.pack_scale_min(sc, mn)[0]
    for j in range(4, 8):
        assert oracle.scale_min(b, j) == (int(sc[0, j]), int(mn[0, j]))


def test_rne_matches_numpy(oracle):
    rng = np.random.default_rng(3)
    bits = np.concatenate([
        rng.integers(0, 2 ** 32, 50_000, dtype=np.uint64).astype(np.uint32),
        np.arange(0x477FE000, 0x47800100, 7, dtype=np.uint32),      # around the overflow threshold 65520
        np.arange(0x387FF000, 0x38801000, 3, dtype=np.uint32),      # subnormal / normal boundary
        np.arange(0x32FFFF00, 0x33000100, dtype=np.uint32),         # 2^-25 tie to zero
        np.array([0, 0x80000000, 0x7F800000, 0xFF800000, 0x7FC00000], dtype=np.uint32),
    ])
    vals = bits.view(np.float32)
    with np.errstate(all="ignore"):
        ref = vals.astype(np.float16).view(np.uint16)
    mine = np.array([oracle.f32_to_f16_rne(float(v)) for v in vals], dtype=np.uint16)
    assert _f16_equal(mine, ref)


def test_gemv_c0_matches_golden(oracle, golden_dir):
    d = np.load(golden_dir / "gemv_c0.npz")
    M, N = int(d["M"]), int(d["N"])
    w = synth.q4k_matrix(M, N, synth.seed_for(0, 0))
    x = synth.activations(1, N, synth.seed_for(0, 100))
    assert hashlib.sha256(w.tobytes()).digest() == d["w_sha256"].tobytes(), "synthetic generator changed"
    assert hashlib.sha256(x.tobytes()).digest() == d["x_sha256"].tobytes()
    y = oracle.q4k_gemv(w, x, M, N)
    _, wn = oracle.q4k_gemv_f64(w, x, M, N)
    ok, ratio, l2 = oracle.tolerance_ok(y, d["y"][None, :], wn, x)
    assert ok and l2 <= 1e-6, (ratio, l2)


def test_gemv_batch_and_threads_consistent(oracle):
    M, N = 96, 512
    w = synth.q4k_matrix(M, N, 1)
    x = synth.activations(3, N, 2)
    y1 = oracle.q4k_gemv(w, x, M, N, threads=1)
    y8 = oracle.q4k_gemv(w, x, M, N, threads=8)
    assert np.array_equal(y1, y8)
    for b in range(3):
        assert np.array_equal(oracle.q4k_gemv(w, x[b], M, N)[0], y1[b])
    # fused decode + dot equals dequant_f16 + matmul_quant on the f16 buffer
    w16 = oracle.dequant_f16(w)
    assert np.array_equal(oracle.matmul_quant_f16(w16, x, M, N), y1)


def test_select_matches_golden(oracle, golden_dir):
    g = np.load(golden_dir / "select.npz")
    for case in ("plain", "ties", "nan", "floor", "ragged", "tiny"):
        v = g[f"{case}_logits"]
        assert oracle.argmax(v) == int(g[f"{case}_argmax"]), case
        vals, idx = oracle.topk256(v)
        assert np.array_equal(vals.view(np.uint32), g[f"{case}_vals"].view(np.uint32)), case
        assert np.array_equal(idx, g[f"{case}_idx"]), case


def test_argmax_tie_rule_follows_the_tree(oracle):
    # The tree of shaders/argmax.wgsl:21-27 moves a value to the lower lane only
    # when strictly greater, so tied residues meet at their lowest differing
    # bit and the one with a 0 there wins (bit-reversed lane order), not the
    # lowest index or the lowest residue.
    v = np.zeros(1024, dtype=np.float32)
    v[[513, 258]] = 5.0        # residues 1 and 2: residue 2 wins (bit 0 clear)
    assert oracle.argmax(v) == 258
    v = np.zeros(1024, dtype=np.float32)
    v[[3, 5]] = 5.0            # residues 3 (011) and 5 (101): lowest differing bit 1 -> 5
    assert oracle.argmax(v) == 5
    v = np.zeros(1024, dtype=np.float32)
    v[[256 + 7, 7]] = 5.0      # same residue: the first (lower) index
    assert oracle.argmax(v) == 7


def test_softcap_and_gelu(oracle):
    x = np.linspace(-1000, 1000, 4001, dtype=np.float32)
    s = oracle.logit_softcap(x, 30.0)
    ref = (np.tanh(np.clip(x.astype(np.float64) / 30.0, -15, 15)) * 30.0)
    assert np.max(np.abs(s - ref)) < 1e-5
    g = np.linspace(-8, 8, 1001, dtype=np.float32)
    u = np.linspace(2, -2, 1001, dtype=np.float32)
    gd = g.astype(np.float64)
    ref = 0.5 * gd * (1 + np.tanh(np.clip(0.7978845608028654 * gd * (1 + 0.044715 * gd * gd), -15, 15))) * u
    assert np.max(np.abs(oracle.gelu_mul(g, u) - ref)) < 1e-5


# ---- Q6_K (src/gguf.ts:316-368) ----------------------------------------------

def test_q6k_dequant_f32_matches_gguf_py(oracle, golden_dir):
    g = np.load(golden_dir / "q6k_blocks.npz")
    out = oracle.q6k_dequant_f32(g["blocks"])
    ref = g["f32"]
    assert np.array_equal(np.isnan(out), np.isnan(ref))
    m = ~np.isnan(ref)
    assert np.array_equal(out[m].view(np.uint32), ref[m].view(np.uint32))


def test_q6k_dequant_f16_matches_golden(oracle, golden_dir):
    g = np.load(golden_dir / "q6k_blocks.npz")
    assert _f16_equal(oracle.q6k_dequant_f16(g["blocks"]), g["f16"])


def test_q6k_known_answer_positions(oracle):
    """d = 1, every scale 1: element 128h + 32s + l is quant s of column l of
    half h (4 bits of ql, 2 bits of qh) minus 32."""
    rng = np.random.default_rng(3)
    b = np.zeros(210, dtype=np.uint8)
    ql = rng.integers(0, 256, 128, dtype=np.uint8)
    qh = rng.integers(0, 256, 64, dtype=np.uint8)
    b[0:128], b[128:192] = ql, qh
    b[192:208] = 1
    b[208:210] = np.array([1.0], dtype=np.float16).view(np.uint8)
    w = oracle.q6k_dequant_f32(b)
    for h in range(2):
        for l in range(32):
            lo0, lo1, hb = int(ql[64 * h + l]), int(ql[64 * h + 32 + l]), int(qh[32 * h + l])
            q = [(lo0 & 15) | ((hb & 3) << 4), (lo1 & 15) | (((hb >> 2) & 3) << 4),
                 (lo0 >> 4) | (((hb >> 4) & 3) << 4), (lo1 >> 4) | (((hb >> 6) & 3) << 4)]
            for s in range(4):
                assert w[128 * h + 32 * s + l] == q[s] - 32


def test_q6k_scales_are_signed_per_16(oracle):
    b = np.zeros(210, dtype=np.uint8)
    b[0:192] = 0xFF                      # every quant 63 -> 31
    sc = np.arange(-8, 8, dtype=np.int8) * 16
    b[192:208] = sc.view(np.uint8)
    b[208:210] = np.array([0.5], dtype=np.float16).view(np.uint8)
    w = oracle.q6k_dequant_f32(b)
    for j in range(16):
        assert np.all(w[16 * j:16 * j + 16] == np.float32(0.5 * int(sc[j]) * 31))


def test_q6k_gemv_matches_f64(oracle):
    M, N = 64, 512
    w = synth.q6k_matrix(M, N, 5)
    x = synth.activations(2, N, 6)
    y = oracle.q6k_gemv(w, x, M, N)
    y64, wn = oracle.q6k_gemv_f64(w, x, M, N)
    w16 = oracle.q6k_dequant_f16(w).view(np.float16).astype(np.float64).reshape(M, N)
    assert np.allclose(y64, x.astype(np.float64) @ w16.T, rtol=1e-12, atol=1e-12)
    assert np.allclose(wn, np.linalg.norm(w16, axis=1))
    assert np.all(np.abs(y - y64) <= 1e-5 * wn[None, :] * np.linalg.norm(x, axis=1)[:, None])


# ---- Q5_K and the per-layer embedding stage 1 --------------------------------
# (src/gguf.ts:212-314, src/engine.ts:642-721, shaders/ple_stage1_fuse.wgsl)

def test_q5k_dequant_f32_matches_gguf_py(oracle, golden_dir):
    g = np.load(golden_dir / "q5k_blocks.npz")
    out = oracle.q5k_dequant_f32(g["blocks"])
    ref = g["f32"]
    assert np.array_equal(np.isnan(out), np.isnan(ref))
    m = ~np.isnan(ref)
    assert np.array_equal(out[m].view(np.uint32), ref[m].view(np.uint32))


def test_q5k_dequant_f16_matches_golden(oracle, golden_dir):
    g = np.load(golden_dir / "q5k_blocks.npz")
    assert _f16_equal(oracle.q5k_dequant_f16(g["blocks"]), g["f16"])


def test_q5k_known_answer_positions(oracle):
    """d = 1, dmin = 0, every scale 1: element 64g + 32h + l is the low (h=0)
    or high (h=1) nibble of qs[32g + l] plus 16 when bit 2g+h of qh[l] is set."""
    rng = np.random.default_rng(4)
    b = np.zeros(176, dtype=np.uint8)
    b[0:2] = np.array([1.0], dtype=np.float16).view(np.uint8)
    b[4:16] = synth.pack_scale_min(np.ones((1, 8), np.uint8), np.zeros((1, 8), np.uint8))[0]
    qh = rng.integers(0, 256, 32, dtype=np.uint8)
    qs = rng.integers(0, 256, 128, dtype=np.uint8)
    b[16:48], b[48:176] = qh, qs
    w = oracle.q5k_dequant_f32(b)
    for g in range(4):
        for h in range(2):
            for l in range(32):
                nib = (int(qs[32 * g + l]) >> (4 * h)) & 15
                q = nib + (16 if (int(qh[l]) >> (2 * g + h)) & 1 else 0)
                assert w[64 * g + 32 * h + l] == q


def test_ple_stage1_oracle_matches_numpy(oracle):
    """The oracle's PLE stage 1 against a float64 statement of the shader's
    formula on the same f16 embedding values: equal to f32 rounding."""
    vocab, layers, T = 16, 5, 3
    table = synth.q5k_table(vocab, layers, 21)
    tokens = np.array([0, 15, 7], dtype=np.uint32)
    rng = np.random.default_rng(22)
    proj = rng.standard_normal((T, layers * 256)).astype(np.float32)
    nw = rng.uniform(0.5, 1.5, 256).astype(np.float16)
    out = oracle.ple_stage1(table, tokens, layers, proj, nw.view(np.uint16), 1e-6)
    emb = oracle.q5k_dequant_f16(table).view(np.float16).astype(np.float64).reshape(vocab, layers, 256)
    for t in range(T):
        for L in range(layers):
            p = proj[t, 256 * L:256 * (L + 1)].astype(np.float64)
            rms = np.sqrt(np.sum(p * p) / 256 + 1e-6)
            ref = (p / rms * nw.astype(np.float64) + emb[tokens[t], L] * 16.0) / np.sqrt(2.0)
            got = out[t, 256 * L:256 * (L + 1)]
            assert np.allclose(got, ref, rtol=2e-6, atol=1e-6)
