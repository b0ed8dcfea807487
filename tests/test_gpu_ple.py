"""GPU parity of the per-layer embedding path (libq4k.so through the C ABI):
the Q5_K table decode against gguf-py's golden vectors and the CPU oracle,
and the fused stage 1 (shaders/ple_stage1_fuse.wgsl over every layer of T
tokens, src/engine.ts:1528-1535) against the oracle's restatement.

Tolerances: decoded f16 values bit-exact (NaN positions matched); stage-1
outputs bit-exact against the oracle (same f32 operations in the same
order, no FMA contraction on either side), checked as at most 1 ulp so a
libm/CUDA square-root difference would show as a clear failure rather than
hide.
"""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from q4k import synth  # noqa: E402
from q4k._lib import Q4KError  # noqa: E402

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
LAYERS = 35  # Gemma-4-E2B num_layers (src/config/gemma4-e2b.ts)


def to_dev(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def _f16_equal(a: np.ndarray, b: np.ndarray) -> bool:
    a, b = a.view(np.uint16), b.view(np.uint16)
    nan_a = ((a & 0x7C00) == 0x7C00) & ((a & 0x3FF) != 0)
    nan_b = ((b & 0x7C00) == 0x7C00) & ((b & 0x3FF) != 0)
    return bool(np.array_equal(nan_a, nan_b) and np.array_equal(a[~nan_a], b[~nan_b]))


def _ulps(a: np.ndarray, b: np.ndarray) -> int:
    ia = a.view(np.int32).astype(np.int64)
    ib = b.view(np.int32).astype(np.int64)
    ia = np.where(ia < 0, -(ia & 0x7FFFFFFF), ia)
    ib = np.where(ib < 0, -(ib & 0x7FFFFFFF), ib)
    return int(np.max(np.abs(ia - ib)))


def test_q5k_dequant_bit_exact_golden(ctx, golden_dir):
    g = np.load(golden_dir / "q5k_blocks.npz")
    out = ctx.q5k_dequant_f16(to_dev(g["blocks"].reshape(-1))).cpu().numpy()
    assert _f16_equal(out, g["f16"])


def test_q5k_dequant_bit_exact_table(ctx, oracle):
    table = synth.q5k_table(64, LAYERS, 31)
    out = ctx.q5k_dequant_f16(to_dev(table.reshape(-1))).cpu().numpy()
    assert _f16_equal(out, oracle.q5k_dequant_f16(table))


def _case(vocab: int, T: int, seed: int):
    rng = np.random.default_rng(seed)
    table = synth.q5k_table(vocab, LAYERS, seed)
    tokens = rng.integers(0, vocab, T).astype(np.uint32)
    tokens[0], tokens[-1] = 0, vocab - 1  # first and last rows of the table
    proj = rng.standard_normal((T, LAYERS * 256)).astype(np.float32)
    nw = rng.uniform(0.25, 2.0, 256).astype(np.float16).view(np.uint16)
    return table, tokens, proj, nw


@pytest.mark.parametrize("T", [1, 4])
def test_ple_stage1_matches_oracle(ctx, oracle, T):
    vocab = 96
    table, tokens, proj, nw = _case(vocab, T, 40 + T)
    out = ctx.ple_stage1(to_dev(table), to_dev(tokens.view(np.int32)), vocab, LAYERS, to_dev(proj),
                         to_dev(nw.view(np.int16)), 1e-6).cpu().numpy()
    ref = oracle.ple_stage1(table, tokens, LAYERS, proj, nw, 1e-6)
    assert np.all(np.isfinite(out))
    assert _ulps(out, ref) <= 1


def test_ple_stage1_zero_projection_and_large_eps(ctx, oracle):
    """A zero projection makes the normalised term exactly 0 (rms = sqrt(eps)):
    the output is the embedding value * 16 / sqrt(2)."""
    vocab = 8
    table, tokens, proj, nw = _case(vocab, 2, 77)
    proj[:] = 0.0
    for eps in (1e-6, 0.5):
        out = ctx.ple_stage1(to_dev(table), to_dev(tokens.view(np.int32)), vocab, LAYERS, to_dev(proj),
                             to_dev(nw.view(np.int16)), eps).cpu().numpy()
        ref = oracle.ple_stage1(table, tokens, LAYERS, proj, nw, eps)
        assert _ulps(out, ref) <= 1


def test_ple_stage1_reads_token_from_device_argmax(ctx, oracle):
    """The token id can come straight from the LM head's argmax output on the
    device (the next forward reads it, src/engine.ts:1719-1727)."""
    V, N, vocab = 4096, 1536, 4096
    wl = synth.q4k_matrix(V, N, 55)
    x = synth.activations(1, N, 56)[0]
    sel = ctx.lmhead_select(to_dev(wl), to_dev(x), V, N, 30.0)
    table, _, proj, nw = _case(vocab, 1, 57)
    out = ctx.ple_stage1(to_dev(table), sel.argmax, vocab, LAYERS, to_dev(proj), to_dev(nw.view(np.int16)),
                         1e-6).cpu().numpy()
    token = np.array([int(sel.argmax.cpu()[0])], dtype=np.uint32)
    ref = oracle.ple_stage1(table, token, LAYERS, proj, nw, 1e-6)
    assert _ulps(out, ref) <= 1


def test_ple_stage1_rejects_token_past_vocab(ctx):
    vocab = 8
    table, _, proj, nw = _case(vocab, 2, 91)
    tokens = np.array([3, vocab], dtype=np.int32)  # the second id is out of range
    out = ctx.ple_stage1(to_dev(table), to_dev(tokens), vocab, LAYERS, to_dev(proj), to_dev(nw.view(np.int16)), 1e-6)
    with pytest.raises(Q4KError):
        ctx.check()
    o = out.cpu().numpy()
    assert np.all(np.isfinite(o[0])) and np.all(np.isnan(o[1]))
    ctx.check()  # the record was cleared
