"""GPU parity of the Q6_K path (libq4k.so through the C ABI) against the CPU
oracle (oracle/q4k_oracle.c restating src/gguf.ts:316-368 + f32ToF16Array +
shaders/matmul_quant.wgsl).

Tolerances as for Q4_K: per output |y - y_ref| <= 1e-3*|y_ref| +
1e-6*||w_row||*||x||, L2 relative error <= 1e-4; weights bit-exact (signed
zeros, infinities and NaN included) through the weight probe.
"""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from q4k import synth  # noqa: E402

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
L2_TOL = 1e-4


def to_dev(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def planar_layout(w: np.ndarray, M: int, N: int) -> np.ndarray:
    """numpy statement of the device layout: bodies [M][nb][208], then the d
    plane [nb][M rounded up to 8] (zero padded)."""
    nb = N // 256
    blocks = w.reshape(M, nb, 210)
    bodies = blocks[:, :, :208].reshape(-1)
    mp = (M + 7) // 8 * 8
    d = np.zeros((nb, mp), dtype=np.uint16)
    d[:, :M] = blocks[:, :, 208:210].copy().view(np.uint16).reshape(M, nb).T
    return np.concatenate([bodies, d.reshape(-1).view(np.uint8)])


def f16_equal(a: np.ndarray, b: np.ndarray) -> bool:
    nan_a = ((a & 0x7C00) == 0x7C00) & ((a & 0x3FF) != 0)
    nan_b = ((b & 0x7C00) == 0x7C00) & ((b & 0x3FF) != 0)
    return np.array_equal(nan_a, nan_b) and np.array_equal(a[~nan_a], b[~nan_b])


def check_gemv(oracle, y_gpu, w, x, M, N):
    y_ref = oracle.q6k_gemv(w, x, M, N)
    _, wn = oracle.q6k_gemv_f64(w, x, M, N)
    ok, ratio, l2 = oracle.tolerance_ok(y_gpu.reshape(y_ref.shape), y_ref, wn, x)
    assert ok, f"per-output bound exceeded: worst ratio {ratio:.3g}"
    assert l2 <= L2_TOL, f"L2 relative {l2:.3g}"


@pytest.mark.parametrize("M,N", [(37, 256), (64, 1536), (300, 512)])
def test_repack_layout(ctx, M, N):
    w = synth.q6k_matrix(M, N, 100 + M)
    dev = ctx.q6k_repack(to_dev(w), M, N)
    assert dev.numel() == ctx.q6k_device_bytes(M, N)
    assert np.array_equal(dev.cpu().numpy(), planar_layout(w, M, N))


def test_probe_bit_exact_golden(ctx, oracle, golden_dir):
    g = np.load(golden_dir / "q6k_blocks.npz")
    blocks = g["blocks"]
    M = blocks.shape[0]  # one super-block per row
    dev = ctx.q6k_repack(to_dev(blocks.reshape(-1)), M, 256)
    out = ctx.q6k_dequant_f16(dev, M, 256).cpu().numpy().view(np.uint16).reshape(-1)
    assert f16_equal(out, g["f16"])
    assert f16_equal(out, oracle.q6k_dequant_f16(blocks))


def test_probe_bit_exact_matrix(ctx, oracle):
    M, N = 200, 1536
    w = synth.q6k_matrix(M, N, 7)
    dev = ctx.q6k_repack(to_dev(w), M, N)
    out = ctx.q6k_dequant_f16(dev, M, N).cpu().numpy().view(np.uint16).reshape(-1)
    assert np.array_equal(out, oracle.q6k_dequant_f16(w))


@pytest.mark.parametrize("M,N,B", [(2048, 1536, 1), (2048, 1536, 3), (1000, 512, 4), (512, 256, 2),
                                   (1536, 6144, 1), (4096, 1536, 7), (256, 2048, 16)])
def test_gemv_matches_oracle(ctx, oracle, M, N, B):
    w = synth.q6k_matrix(M, N, M + N + B)
    x = synth.activations(B, N, 9 + B)
    dev = ctx.q6k_repack(to_dev(w), M, N)
    y = ctx.q6k_gemv(dev, to_dev(x), M, N).cpu().numpy()
    check_gemv(oracle, y, w, x, M, N)


def test_gemv_batch_over_16_chunks(ctx, oracle):
    M, N, B = 512, 1536, 21
    w = synth.q6k_matrix(M, N, 77)
    x = synth.activations(B, N, 78)
    dev = ctx.q6k_repack(to_dev(w), M, N)
    check_gemv(oracle, ctx.q6k_gemv(dev, to_dev(x), M, N).cpu().numpy(), w, x, M, N)


def test_gemv_non_finite_d_rows(ctx, oracle):
    """Rows whose d is inf or NaN take the exact decode: the same inf/NaN
    outputs as the reference's f16 weights give; other rows are unaffected."""
    M, N = 64, 512
    w = synth.q6k_matrix(M, N, 5).copy()
    blk = w.reshape(M, 2, 210)
    blk[3, 1, 208:210] = np.array([0x7C00], dtype=np.uint16).view(np.uint8)  # +inf
    blk[10, 0, 208:210] = np.array([0x7E00], dtype=np.uint16).view(np.uint8)  # NaN
    x = synth.activations(1, N, 6)
    dev = ctx.q6k_repack(to_dev(w), M, N)
    y = ctx.q6k_gemv(dev, to_dev(x), M, N).cpu().numpy()[0]
    y_ref = oracle.q6k_gemv(w, x, M, N)[0]
    bad = np.array([3, 10])
    assert np.array_equal(np.isnan(y[bad]), np.isnan(y_ref[bad]))
    assert np.array_equal(np.isinf(y[bad]), np.isinf(y_ref[bad]))
    good = np.setdiff1d(np.arange(M), bad)
    _, wn = oracle.q6k_gemv_f64(w, x, M, N)
    ok, ratio, _ = oracle.tolerance_ok(y[good][None], y_ref[good][None], wn[good], x)
    assert ok, ratio


def test_lmhead_select_q6k(ctx, oracle):
    V, N = 65536, 1536
    w = synth.q6k_matrix(V, N, 4242)
    x = synth.activations(1, N, 4243)
    dev = ctx.q6k_repack(to_dev(w), V, N)
    sel = ctx.q6k_lmhead_select(dev, to_dev(x[0]), V, N, 30.0, return_logits=True)
    torch.cuda.synchronize()
    logits = oracle.logit_softcap(oracle.q6k_gemv(w, x, V, N)[0], 30.0)
    gl = sel.logits.cpu().numpy()
    assert np.linalg.norm(gl - logits) / np.linalg.norm(logits) <= L2_TOL
    top2 = np.sort(logits)[-2:]
    if top2[1] - top2[0] > 2e-3:
        assert int(sel.argmax.cpu()[0]) == oracle.argmax(logits)
    buf = ctx.topk256(sel.logits).cpu().numpy()
    assert np.array_equal(buf[1::2].view(np.uint32), sel.cand_idx.cpu().numpy().view(np.uint32))
    assert np.array_equal(buf[0::2].view(np.uint32), sel.cand_val.cpu().numpy().view(np.uint32))
    assert int(ctx.argmax(sel.logits).cpu()[0]) == int(sel.argmax.cpu()[0])
    # candidate indices agree with the oracle's per-residue maxima except near-ties
    ref_val = np.full(256, -1e30, np.float32)
    ref_idx = np.zeros(256, np.int64)
    for r in range(256):
        v = logits[r::256]
        i = int(np.argmax(v))
        ref_val[r], ref_idx[r] = v[i], r + 256 * i
    gi = sel.cand_idx.cpu().numpy().astype(np.int64)
    mism = np.nonzero(gi != ref_idx)[0]
    for r in mism:
        assert abs(logits[gi[r]] - ref_val[r]) <= 2e-3


def test_gguf_q6k_tensor_probe(ctx, oracle, golden_dir):
    from q4k import gguf as G

    f = G.open_gguf(golden_dir / "tiny_q4k.gguf")
    dev, M, N = G.upload_q6k(f, "blk.0.q6_k.weight", ctx)
    raw = np.array(f.q6k_matrix("blk.0.q6_k.weight")[0])
    out = ctx.q6k_dequant_f16(dev, M, N).cpu().numpy().view(np.uint16).reshape(-1)
    assert f16_equal(out, oracle.q6k_dequant_f16(raw))


def test_q6k_rejects_bad_arguments(ctx):
    from q4k import Q4KError

    w = torch.zeros(ctx.q6k_device_bytes(16, 256) + 16, dtype=torch.uint8, device=DEV)
    x = torch.zeros(256, dtype=torch.float32, device=DEV)
    with pytest.raises(ValueError):
        ctx.q6k_gemv(w, x, 16, 100)
    with pytest.raises(Q4KError):
        ctx.q6k_gemv(w[1:], x, 16, 256)  # misaligned weights
    g = torch.zeros(2 * 210 * 16 + 2, dtype=torch.uint8, device=DEV)
    with pytest.raises(Q4KError):
        ctx.q6k_repack(g[1:1 + 2 * 210 * 16], 16, 256 * 2)  # odd GGUF pointer


def test_plan_mixed_formats_match_single_calls(ctx):
    """A stage mixing Q4_K and Q6_K GEMVs (sharing an input) and a Q6_K LM
    head, then a gelu_mul feeding a Q6_K down projection: the plan's outputs
    equal the single calls' (same kernels, same per-output arithmetic)."""
    from q4k import Plan

    N, M, I, V = 1536, 2048, 6144, 16384
    wq = to_dev(synth.q4k_matrix(M, N, 1))
    wv = ctx.q6k_repack(to_dev(synth.q6k_matrix(512, N, 2)), 512, N)
    wg = to_dev(synth.q4k_matrix(I, N, 3))
    wd = ctx.q6k_repack(to_dev(synth.q6k_matrix(N, I, 4)), N, I)
    wh = ctx.q6k_repack(to_dev(synth.q6k_matrix(V, N, 5)), V, N)
    x = to_dev(synth.activations(1, N, 6)[0])
    gate = to_dev(synth.activations(1, I, 7)[0])
    up = to_dev(synth.activations(1, I, 8)[0])
    yq = torch.empty(M, device=DEV)
    yv = torch.empty(512, device=DEV)
    yg = torch.empty(I, device=DEV)
    act = torch.empty(I, device=DEV)
    yd = torch.empty(N, device=DEV)
    from q4k import Selection
    sel = Selection(torch.empty(256, device=DEV), torch.empty(256, dtype=torch.int32, device=DEV),
                    torch.empty(1, dtype=torch.int32, device=DEV), torch.empty(V, device=DEV))
    p = Plan(ctx, 1)
    p.gemv(0, wq, x, yq, M, N)
    p.gemv_q6k(0, wv, x, yv, 512, N)
    p.gemv(0, wg, x, yg, I, N)
    p.lmhead_q6k(0, wh, x, V, N, 30.0, sel)
    p.gelu_mul(1, gate, up, act)
    p.gemv_q6k(1, wd, act, yd, N, I)
    p.commit()
    assert p.launches() == 3  # stage 0: a Q4_K and a Q6_K launch; stage 1: one Q6_K launch
    p.run()
    torch.cuda.synchronize()
    assert torch.equal(yq, ctx.gemv(wq, x, M, N)[0])
    assert torch.equal(yv, ctx.q6k_gemv(wv, x, 512, N)[0])
    assert torch.equal(yg, ctx.gemv(wg, x, I, N)[0])
    ref_act = ctx.gelu_mul(gate, up)
    assert torch.equal(act, ref_act)
    assert torch.equal(yd, ctx.q6k_gemv(wd, ref_act, N, I)[0])
    ref = ctx.q6k_lmhead_select(wh, x, V, N, 30.0, return_logits=True)
    assert torch.equal(sel.logits, ref.logits)
    assert torch.equal(sel.cand_idx, ref.cand_idx) and torch.equal(sel.argmax, ref.argmax)


def test_real_e2b_step_plan_matches_serial(ctx, oracle):
    """The real-shape step (full-attention and sliding layers, producer and
    consumer layers, Q4_K/Q6_K mix, PLE GEMVs, Q6_K LM head) through the plan
    equals the one-call-per-dispatch order, and two of its GEMVs match the
    oracle."""
    from q4k.e2b import FMT_Q6K, RealE2BStep, layer_matrices, matrix_host, MAT_IDS, CONFIG

    step = RealE2BStep(ctx, layers=(0, 4, 15, 34))
    step.run()
    torch.cuda.synchronize()
    got = {k: v.clone() for k, v in step.out.items()}
    sel = (step.sel.cand_idx.clone(), step.sel.argmax.clone())
    ple = step.ple_out.clone()
    ple_in = step.ple_inputs.clone()
    # two stages x two formats, each engine launch preceded by a preparation
    # launch when its CTAs cannot cache all of their activations
    assert 4 <= step.plan().launches() <= 8
    step.run_serial()
    torch.cuda.synchronize()
    for k in got:
        M, N, fmt, _ = step.mats[k]
        if k[1] == "down" or (fmt != FMT_Q6K and N // 256 >= 16):
            # long rows split each tile's K range over 4 warps (partial sums
            # added in order) in a stage of downs and in single calls: the
            # same products, another order
            d = (got[k] - step.out[k]).norm() / step.out[k].norm()
            assert d <= 2e-5, (k, float(d))
        else:
            assert torch.equal(got[k], step.out[k]), k
    assert torch.equal(sel[0], step.sel.cand_idx) and torch.equal(sel[1], step.sel.argmax)
    assert torch.equal(ple, step.ple_out)
    assert torch.equal(ple_in, step.ple_inputs)
    # the per-layer embedding stage 1 of the chosen token, read from the Q5_K
    # table on the device, against the oracle on that token's table row
    tok = int(step.sel.argmax.cpu()[0])
    row = step.ple_table[tok].cpu().numpy()[None]
    ref = oracle.ple_stage1(row, np.zeros(1, dtype=np.uint32), step.shape.layers, ple.cpu().numpy()[None],
                            step.ple_norm.cpu().numpy().view(np.uint16), 1e-6)
    assert np.max(np.abs(ple_in.cpu().numpy() - ref[0]) / (np.abs(ref[0]) + 1e-30)) <= 2.5e-7
    # layer 0's v and down are Q6_K, layer 4's q is 4096 x 1536 Q4_K, layer
    # 15's down is 1536 x 12288 Q4_K (the plan's outputs, K-split downs included)
    for (layer, name) in ((0, "v"), (4, "q"), (0, "down"), (15, "down")):
        M, N, fmt, _ = layer_matrices(step.shape, layer)[name]
        if name == "v" or (layer, name) == (0, "down"):
            assert fmt == FMT_Q6K
        w = matrix_host(M, N, fmt, synth.seed_for(CONFIG, 16 * layer + MAT_IDS.index(name)))
        x = (step.act[layer] if name == "down" else step.x["h"]).cpu().numpy()[None]
        ref = oracle.q6k_gemv(w, x, M, N) if fmt == FMT_Q6K else oracle.q4k_gemv(w, x, M, N)
        _, wn = (oracle.q6k_gemv_f64 if fmt == FMT_Q6K else oracle.q4k_gemv_f64)(w, x, M, N)
        ok, ratio, l2 = oracle.tolerance_ok(got[(layer, name)].cpu().numpy()[None], ref, wn, x)
        assert ok and l2 <= L2_TOL, (layer, name, ratio, l2)
