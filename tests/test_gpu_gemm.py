"""GPU parity of the batched Q4_K GEMM (q4k_gemm, tcgen05) against the oracle.

Same tolerance as the GEMV (per output 1e-3*|y_ref| + 1e-6*||w_row||*||x||,
L2 relative 1e-4): the weights are the reference's f16 values exactly and x
enters the tensor core split into exact f16 hi + lo parts, so only the fp32
accumulation order differs from the oracle's.

q4k_gemm_f16x rounds each scaled activation row once to f16.  Against the
oracle on the f32 activations it meets the prefill tolerance (L2 relative
2e-3; per output 2e-3*|y_ref| + 1e-4*||w_row||*||x||); against the oracle
on the same f16-rounded activations it meets the GEMV tolerance above.
"""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from q4k import synth  # noqa: E402

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def to_dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def check(oracle, y, w, x, M, N):
    y_ref = oracle.q4k_gemv(w, x, M, N)
    _, wn = oracle.q4k_gemv_f64(w, x, M, N)
    ok, ratio, l2 = oracle.tolerance_ok(y.reshape(y_ref.shape), y_ref, wn, x)
    assert ok, f"per-output bound exceeded: worst ratio {ratio:.3g}"
    assert l2 <= 1e-4, f"L2 relative {l2:.3g}"


@pytest.mark.parametrize("M,N,T", [
    (128, 256, 64), (256, 1536, 64), (300, 768, 100), (2048, 1536, 128), (1536, 2048, 200),
    (130, 6144, 65), (1024, 1536, 512), (64, 512, 1), (200, 1024, 17), (6144, 1536, 512),
])
def test_gemm_shapes(ctx, oracle, M, N, T):
    w = synth.q4k_matrix(M, N, synth.seed_for(4, M + N))
    x = synth.activations(T, N, synth.seed_for(4, 700 + T))
    y = ctx.gemm(to_dev(w), to_dev(x), M, N).cpu().numpy()
    check(oracle, y, w, x, M, N)


def f16_rounded(x: np.ndarray) -> np.ndarray:
    """Each row of x scaled by the GEMM's power of two (max|x_t| * s < 2^15),
    rounded to f16 and scaled back: the activations q4k_gemm_f16x multiplies."""
    out = np.empty_like(x)
    for t in range(x.shape[0]):
        mx = float(np.max(np.abs(x[t])))
        sexp = 0
        if mx > 0.0:
            sexp = int(np.clip(15 - np.frexp(mx)[1], -100, 100))
        s = np.float32(2.0 ** sexp)
        out[t] = (x[t] * s).astype(np.float16).astype(np.float32) / s
    return out


@pytest.mark.parametrize("M,N,T", [
    (256, 1536, 64), (300, 768, 100), (2048, 1536, 256), (1536, 2048, 257), (130, 6144, 65),
    (1024, 1536, 512), (64, 512, 1), (200, 1024, 17), (6144, 1536, 600),
])
def test_gemm_f16x_shapes(ctx, oracle, M, N, T):
    w = synth.q4k_matrix(M, N, synth.seed_for(4, M + N + 1))
    x = synth.activations(T, N, synth.seed_for(4, 900 + T))
    y = ctx.gemm(to_dev(w), to_dev(x), M, N, f16x=True).cpu().numpy()
    # exactly the f16-rounded activations, up to accumulation order
    check(oracle, y, w, f16_rounded(x), M, N)
    # and within the prefill tolerance of the f32 activations
    y_ref = oracle.q4k_gemv(w, x, M, N)
    _, wn = oracle.q4k_gemv_f64(w, x, M, N)
    y = y.reshape(y_ref.shape)
    l2 = float(np.linalg.norm(y - y_ref) / np.linalg.norm(y_ref))
    assert l2 <= 2e-3, f"L2 relative {l2:.3g}"
    bound = 2e-3 * np.abs(y_ref) + 1e-4 * wn[None, :] * np.linalg.norm(x, axis=1)[:, None]
    assert np.all(np.abs(y - y_ref) <= bound)


def test_gemv_hands_large_batches_to_the_gemm(ctx, oracle):
    M, N, T = 512, 1536, 96
    w = synth.q4k_matrix(M, N, 91)
    x = synth.activations(T, N, 92)
    wd, xd = to_dev(w), to_dev(x)
    y_gemv = ctx.gemv(wd, xd, M, N)
    y_gemm = ctx.gemm(wd, xd, M, N)
    torch.cuda.synchronize()
    assert torch.equal(y_gemv.view(torch.int32), y_gemm.view(torch.int32))
    check(oracle, y_gemv.cpu().numpy(), w, x, M, N)


def test_gemm_repeatable_and_leaves_neighbours(ctx):
    M, N, T = 384, 1536, 130
    w = to_dev(synth.q4k_matrix(M, N, 93))
    x = to_dev(synth.activations(T, N, 94))
    canary = torch.full((T * M + 64,), 7.25, dtype=torch.float32, device=DEV)
    y = canary[:T * M].view(T, M)
    ctx.gemm(w, x, M, N, out=y)
    first = y.clone()
    ctx.gemm(w, x, M, N, out=y)
    torch.cuda.synchronize()
    assert torch.equal(first.view(torch.int32), y.view(torch.int32))
    assert torch.all(canary[T * M:] == 7.25)
    ctx.check()


def test_batched_sweep_streams_match_single_calls(ctx):
    """Config 4's GEMM path spreads the layers over several streams, each with
    its own library context: every output equals a single q4k_gemm call on
    the default stream, bit for bit."""
    from q4k.decode import BatchedSweep, DecodeStep, E2BShape, layer_shapes

    step = DecodeStep(ctx, E2BShape(layers=3, vocab=1024))
    bs = BatchedSweep(step, 64, streams=2, exact=True, mode="streams")
    bs.run()
    torch.cuda.synchronize()
    shapes = layer_shapes(step.shape)
    for layer in range(3):
        for name, (M, N) in shapes.items():
            x = bs.act[layer] if name == "down" else (bs.x_attn if name == "o" else bs.x_h)
            ref = ctx.gemm(step.weights[(layer, name)], x, M, N)
            torch.cuda.synchronize()
            assert torch.equal(ref.view(torch.int32), bs.out[(layer, name)].view(torch.int32)), (layer, name)
    bs.close()


def test_batched_sweep_f16x_matches_single_calls(ctx):
    from q4k.decode import BatchedSweep, DecodeStep, E2BShape, layer_shapes

    step = DecodeStep(ctx, E2BShape(layers=2, vocab=1024))
    bs = BatchedSweep(step, 300, streams=2, f16x=True, mode="streams")
    bs.run()
    torch.cuda.synchronize()
    shapes = layer_shapes(step.shape)
    for layer in range(2):
        for name, (M, N) in shapes.items():
            x = bs.act[layer] if name == "down" else (bs.x_attn if name == "o" else bs.x_h)
            ref = ctx.gemm(step.weights[(layer, name)], x, M, N, f16x=True)
            torch.cuda.synchronize()
            assert torch.equal(ref.view(torch.int32), bs.out[(layer, name)].view(torch.int32)), (layer, name)
    bs.close()


@pytest.mark.parametrize("T,exact", [(64, True), (64, False), (100, False), (128, False), (300, False), (512, False), (65, True)])
def test_gemm_plan_one_launch_per_stage_matches_oracle(ctx, oracle, T, exact):
    """A batch >= 64 plan runs each stage as one preparation launch plus ONE
    GEMM launch over all its matrices (two layers' q/k/v/o/gate/up, then
    gelu_mul + both downs): every output matches the oracle -- exact plans
    on the f32 activations, f16 plans on the f16-rounded activations -- within
    the GEMV tolerance, and the stored gelu_mul output is the oracle's.  The
    down stage (few tiles) runs K-split; a second run repeats every bit."""
    from q4k.decode import BatchedSweep, DecodeStep, E2BShape, LAYER_MATS, layer_shapes, matrix_seed

    shape = E2BShape(layers=2, vocab=1024)
    step = DecodeStep(ctx, shape)
    bs = BatchedSweep(step, T, exact=exact)
    assert bs.plan is not None and bs.plan.launches() == 4
    bs.run()
    torch.cuda.synchronize()
    ctx.check()
    shapes = layer_shapes(shape)
    x_h, x_attn = bs.x_h.cpu().numpy(), bs.x_attn.cpu().numpy()
    feed = (lambda a: a) if exact else f16_rounded
    for layer in range(2):
        W = {name: synth.q4k_matrix(*shapes[name], matrix_seed(layer, name)) for name in LAYER_MATS}
        out = {name: bs.out[(layer, name)].cpu().numpy() for name in LAYER_MATS}
        for name in ("q", "k", "v", "o", "gate", "up"):
            M, N = shapes[name]
            check(oracle, out[name], W[name], feed(x_attn if name == "o" else x_h), M, N)
        act = bs.act[layer].cpu().numpy()
        act_ref = oracle.gelu_mul(out["gate"], out["up"])
        assert np.all(np.abs(act - act_ref) <= 1e-6 * np.abs(out["gate"] * out["up"]) + 1e-6 * np.abs(act_ref))
        M, N = shapes["down"]
        check(oracle, out["down"], W["down"], feed(act), M, N)
    # a second run gives the same bits: the down stage runs as two K halves
    # accumulated into its zeroed outputs, and 0 + a + b is exact in either
    # order
    first = {key: t.clone() for key, t in bs.out.items()}
    bs.run()
    torch.cuda.synchronize()
    ctx.check()
    for key, t in bs.out.items():
        assert torch.equal(t.view(torch.int32), first[key].view(torch.int32)), key



def test_gemm_plan_wide_rows_take_the_two_pass_preparation(ctx, oracle):
    """A GEMM plan whose activation rows are wider than the single-read
    preparation stages in shared memory (N > 24576 floats) prepares them in
    two passes over global memory instead; the result still matches the
    oracle on the f16-rounded activations within the GEMV tolerance."""
    from q4k import Plan

    T, M, N = 64, 256, 97 * 256
    w = synth.q4k_matrix(M, N, synth.seed_for(4, 97))
    x = synth.activations(T, N, synth.seed_for(4, 98))
    y = torch.zeros(T * M, dtype=torch.float32, device=DEV)
    p = Plan(ctx, T)
    p.gemv(0, to_dev(w), to_dev(x), y, M, N)
    p.commit()
    p.run()
    torch.cuda.synchronize()
    ctx.check()
    check(oracle, y.cpu().numpy().reshape(T, M), w, f16_rounded(x), M, N)
    p.close()
