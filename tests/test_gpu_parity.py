"""GPU parity: libq4k.so kernels (through the C ABI) against the CPU oracle.

Tolerances: per output |y - y_ref| <= 1e-3*|y_ref| +
1e-6*||w_row||*||x||, L2 relative error <= 1e-4; weights, argmax and
candidate index sets bit-exact except near-ties whose gap is inside the f32
summation-order error (both sides accumulate in f32, in different orders).
"""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from q4k import Q4KError, synth  # noqa: E402

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
L2_TOL = 1e-4


def to_dev(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def check_gemv(oracle, y_gpu: np.ndarray, w: np.ndarray, x: np.ndarray, M: int, N: int):
    y_ref = oracle.q4k_gemv(w, x, M, N)
    _, wn = oracle.q4k_gemv_f64(w, x, M, N)
    ok, ratio, l2 = oracle.tolerance_ok(y_gpu.reshape(y_ref.shape), y_ref, wn, x)
    assert ok, f"per-output bound exceeded: worst ratio {ratio:.3g}"
    assert l2 <= L2_TOL, f"L2 relative {l2:.3g}"
    return l2


def test_dequant_f16_bit_exact_golden(ctx, oracle, golden_dir):
    g = np.load(golden_dir / "q4k_blocks.npz")
    out = ctx.dequant_f16(to_dev(g["blocks"].reshape(-1))).cpu().numpy().view(np.uint16)
    ref = g["f16"]
    nan_o = ((out & 0x7C00) == 0x7C00) & ((out & 0x3FF) != 0)
    nan_r = ((ref & 0x7C00) == 0x7C00) & ((ref & 0x3FF) != 0)
    assert np.array_equal(nan_o, nan_r)
    assert np.array_equal(out[~nan_o], ref[~nan_r])


def test_dequant_f16_bit_exact_matrix(ctx, oracle):
    w = synth.q4k_matrix(512, 1536, synth.seed_for(0, 7))
    out = ctx.dequant_f16(to_dev(w.reshape(-1))).cpu().numpy().view(np.uint16)
    assert np.array_equal(out, oracle.dequant_f16(w))


def test_matmul_quant_config0_golden(ctx, oracle, golden_dir):
    d = np.load(golden_dir / "gemv_c0.npz")
    M, N = 2048, 1536
    w = synth.q4k_matrix(M, N, synth.seed_for(0, 0))
    x = synth.activations(1, N, synth.seed_for(0, 100))
    out = torch.empty(M, dtype=torch.float32, device=DEV)
    ctx.matmul_quant(to_dev(x), to_dev(w), out, M, N)
    torch.cuda.synchronize()
    y = out.cpu().numpy()[None, :]
    check_gemv(oracle, y, w, x, M, N)
    _, wn = oracle.q4k_gemv_f64(w, x, M, N)
    ok, ratio, l2 = oracle.tolerance_ok(y, d["y"][None, :], wn, x)
    assert ok and l2 <= L2_TOL, (ratio, l2)


@pytest.mark.parametrize("M,N,batch", [
    (1, 256, 1), (7, 256, 1), (13, 512, 2), (256, 1536, 1), (2048, 1536, 4), (1536, 2048, 1),
    (1536, 6144, 1), (300, 768, 3), (64, 1536, 5), (96, 1536, 8), (40, 2560, 16), (33, 1536, 16),
])
def test_gemv_shapes(ctx, oracle, M, N, batch):
    w = synth.q4k_matrix(M, N, synth.seed_for(9, M + N))
    x = synth.activations(batch, N, synth.seed_for(9, 500 + batch))
    y = ctx.gemv(to_dev(w), to_dev(x), M, N).cpu().numpy()
    check_gemv(oracle, y, w, x, M, N)


def test_gemv_large_m_2d_grid_case(ctx, oracle):
    # M > 65535 (the reference switches to a 2-D grid there, src/engine.ts:332-341).
    M, N = 70_000, 256
    w = synth.q4k_matrix(M, N, 77)
    x = synth.activations(1, N, 78)
    y = ctx.gemv(to_dev(w), to_dev(x), M, N).cpu().numpy()
    check_gemv(oracle, y, w, x, M, N)


def test_gemv_rowwarp_path(ctx, oracle):
    """Requests whose prepared activation (4 bytes per element per row) would
    exceed the context's 16 MB scratch take the scratch-free warp-per-row
    kernel: 16 rows of N = 262400 need 16.8 MB.  batch 19 runs as chunks of
    16 (warp per row) and 3 (the engine with a separate preparation launch)."""
    M, N, batch = 24, 262400, 19
    w = synth.q4k_matrix(M, N, 81)
    x = synth.activations(batch, N, 82)
    y = ctx.gemv(to_dev(w), to_dev(x), M, N).cpu().numpy()
    check_gemv(oracle, y, w, x, M, N)


def test_config1_ffn_chain(ctx, oracle):
    I, H = 6144, 1536
    wg = synth.q4k_matrix(I, H, synth.seed_for(1, 0))
    wu = synth.q4k_matrix(I, H, synth.seed_for(1, 1))
    wd = synth.q4k_matrix(H, I, synth.seed_for(1, 2))
    x = synth.activations(1, H, synth.seed_for(1, 100))
    xd = to_dev(x)
    g = ctx.gemv(to_dev(wg), xd, I, H)
    u = ctx.gemv(to_dev(wu), xd, I, H)
    a = ctx.gelu_mul(g, u)
    y = ctx.gemv(to_dev(wd), a, H, I).cpu().numpy()
    # oracle chain on the oracle's own intermediates
    g_ref = oracle.q4k_gemv(wg, x, I, H)
    u_ref = oracle.q4k_gemv(wu, x, I, H)
    a_ref = oracle.gelu_mul(g_ref, u_ref)
    check_gemv(oracle, g.cpu().numpy(), wg, x, I, H)
    check_gemv(oracle, u.cpu().numpy(), wu, x, I, H)
    # down is checked against the oracle fed with the GPU's activation (same input) ...
    check_gemv(oracle, y, wd, a.cpu().numpy(), H, I)
    # ... and the whole chain against the oracle chain within the L2 bound
    y_ref = oracle.q4k_gemv(wd, a_ref, H, I)
    assert np.linalg.norm(y - y_ref) / np.linalg.norm(y_ref) <= L2_TOL


def test_standalone_select_ops_exact(ctx, golden_dir):
    g = np.load(golden_dir / "select.npz")
    for case in ("plain", "ties", "nan", "floor", "ragged", "tiny"):
        v = to_dev(g[f"{case}_logits"])
        am = int(ctx.argmax(v).cpu().numpy()[0])
        assert am == int(g[f"{case}_argmax"]), case
        buf = ctx.topk256(v).cpu().numpy()
        assert np.array_equal(buf[0::2].view(np.uint32), g[f"{case}_vals"].view(np.uint32)), case
        assert np.array_equal(buf[1::2].view(np.uint32), g[f"{case}_idx"]), case


def test_select_rows_golden_exact(ctx, golden_dir):
    """The batched softcap/topk256/argmax (one launch for all rows) on the
    golden selection cases (ties, NaN, the -1e30 floor, ragged and tiny
    lengths), without a softcap: bit-exact candidates and argmax."""
    g = np.load(golden_dir / "select.npz")
    for case in ("plain", "ties", "nan", "floor", "ragged", "tiny"):
        logits = g[f"{case}_logits"]
        rows = np.stack([logits, logits])  # two identical rows: both must give the golden answer
        cv, ci, am = ctx.select_rows(to_dev(rows), 0.0)
        for b in range(2):
            assert int(am[b].cpu()) == int(g[f"{case}_argmax"]), case
            assert np.array_equal(cv[b].cpu().numpy().view(np.uint32), g[f"{case}_vals"].view(np.uint32)), case
            assert np.array_equal(ci[b].cpu().numpy().view(np.uint32), g[f"{case}_idx"]), case


@pytest.mark.parametrize("B,n", [(1, 262144), (4, 262144), (3, 1000), (16, 4096), (2, 37)])
def test_select_rows_equals_per_row_ops(ctx, B, n):
    """With a softcap: the one-launch form equals q4k_logit_softcap +
    q4k_topk256 + q4k_argmax run row by row, bit for bit (softcapped logits
    included), on rows with planted ties and NaN."""
    rng = np.random.default_rng(B * 1000 + n)
    x = (rng.standard_normal((B, n)) * 40).astype(np.float32)
    x[:, n // 3] = 500.0
    x[:, (2 * n) // 3] = 500.0  # a tie at the top (after the softcap too)
    x[0, n // 2] = np.nan
    got = to_dev(x)
    cv, ci, am = ctx.select_rows(got, 30.0)
    for b in range(B):
        row = to_dev(x[b])
        ctx.logit_softcap(row, 30.0)
        assert torch.equal(row.view(torch.int32), got[b].view(torch.int32)), b
        buf = ctx.topk256(row).cpu().numpy()
        assert np.array_equal(cv[b].cpu().numpy().view(np.uint32), buf[0::2].view(np.uint32)), b
        assert np.array_equal(ci[b].cpu().numpy().view(np.uint32), buf[1::2].view(np.uint32)), b
        assert int(am[b].cpu()) == int(ctx.argmax(row).cpu()[0]), b


def test_select_rows_repeat_calls(ctx):
    """The row scratch is back in its between-calls state after every call."""
    x = torch.randn(4, 5000, device=DEV)
    first = [t.clone() for t in ctx.select_rows(x.clone(), 0.0)]
    for _ in range(3):
        again = ctx.select_rows(x.clone(), 0.0)
        assert all(torch.equal(a, b) for a, b in zip(first, again))


def test_softcap_and_gelu(ctx, oracle):
    rng = np.random.default_rng(4)
    v = (rng.standard_normal(100_000) * 200).astype(np.float32)
    v[:5] = [0.0, -0.0, 1e30, -1e30, 449.9]
    out = ctx.logit_softcap(to_dev(v), 30.0).cpu().numpy()
    ref = oracle.logit_softcap(v, 30.0)
    assert np.max(np.abs(out - ref)) <= 4 * np.spacing(np.float32(30.0))
    gte = (rng.standard_normal(50_000) * 4).astype(np.float32)
    up = rng.standard_normal(50_000).astype(np.float32)
    o = ctx.gelu_mul(to_dev(gte), to_dev(up)).cpu().numpy()
    r = oracle.gelu_mul(gte, up)
    # CUDA tanhf and libm tanhf may differ by a few ulp; that error is
    # relative to 0.5*|gate*up| (the tanh term's scale), not to the result.
    bound = 1e-6 * np.abs(gte * up) + 1e-6 * np.abs(r)
    assert np.all(np.abs(o - r) <= bound)


def _selection_matches(oracle, w, x, V, N, row_offset, sel, cap=30.0, gap_tol=2e-3):
    """Compare a GPU Selection with the oracle's logits -> topk256/argmax."""
    y = oracle.q4k_gemv(w, x, V, N)[0]
    logits = oracle.logit_softcap(y, cap)
    full = np.full(row_offset + V, -3e38, dtype=np.float32)
    full[row_offset:] = logits
    vals_ref, idx_ref = oracle.topk256(full)
    cv = sel.cand_val.cpu().numpy()
    ci = sel.cand_idx.cpu().numpy().view(np.uint32)
    ambiguous = 0
    for r in range(256):
        mem = logits[(np.arange(V) + row_offset) % 256 == r]
        if mem.size == 0:
            continue
        top2 = np.sort(mem)[-2:] if mem.size > 1 else np.array([-np.inf, mem.max()])
        if top2[1] - top2[0] <= gap_tol:
            ambiguous += 1
            assert logits[ci[r] - row_offset] >= top2[1] - gap_tol
            continue
        assert ci[r] == idx_ref[r], f"residue {r}: {ci[r]} vs {idx_ref[r]}"
        assert abs(cv[r] - vals_ref[r]) <= 1e-3, (r, cv[r], vals_ref[r])
    return ambiguous, logits


def test_lmhead_select_config2(ctx, oracle):
    V, N = 262144, 1536
    w = synth.q4k_matrix(V, N, synth.seed_for(2, 0))
    x = synth.activations(1, N, synth.seed_for(2, 100))
    sel = ctx.lmhead_select(to_dev(w), to_dev(x[0]), V, N, 30.0, return_logits=True)
    torch.cuda.synchronize()
    ambiguous, logits = _selection_matches(oracle, w, x, V, N, 0, sel)
    assert ambiguous <= 8
    gl = sel.logits.cpu().numpy()
    assert np.linalg.norm(gl - logits) / np.linalg.norm(logits) <= L2_TOL
    # argmax: exact unless the oracle's top-2 overall gap is inside the error
    top2 = np.sort(logits)[-2:]
    if top2[1] - top2[0] > 2e-3:
        assert int(sel.argmax.cpu()[0]) == oracle.argmax(logits)
    # the fused candidates are exactly what the standalone ops give on the GPU logits
    buf = ctx.topk256(sel.logits).cpu().numpy()
    assert np.array_equal(buf[1::2].view(np.uint32), sel.cand_idx.cpu().numpy().view(np.uint32))
    assert np.array_equal(buf[0::2].view(np.uint32), sel.cand_val.cpu().numpy().view(np.uint32))
    assert int(ctx.argmax(sel.logits).cpu()[0]) == int(sel.argmax.cpu()[0])


@pytest.mark.parametrize("G", [2, 4, 8])
def test_sharded_lmhead_merge_equals_unsharded(ctx, oracle, G):
    V, N = 65536, 512
    w = synth.q4k_matrix(V, N, 4242)
    x = synth.activations(1, N, 4343)
    wd, xd = to_dev(w), to_dev(x[0])
    full = ctx.lmhead_select(wd, xd, V, N, 30.0)
    shard = V // G
    vals, idx = [], []
    for r in range(G):
        s = ctx.lmhead_select(wd[r * shard:(r + 1) * shard], xd, shard, N, 30.0, row_offset=r * shard)
        vals.append(s.cand_val.clone())
        idx.append(s.cand_idx.clone())
    m = ctx.merge_candidates(torch.cat(vals), torch.cat(idx))
    assert torch.equal(m.cand_idx, full.cand_idx)
    assert torch.equal(m.cand_val.view(torch.int32), full.cand_val.view(torch.int32))
    assert torch.equal(m.argmax, full.argmax)


def test_fused_exchange_one_rank_equals_unsharded(ctx):
    # the fused sharded head with a world of 1: the launch writes its
    # candidates into its own mailbox, waits for them and merges.  Calls go
    # back to back with a different input each and no host synchronization
    # in between, so consecutive calls alternate the mailbox's two slot sets
    # (epoch parity) while the previous call's data is still fresh.
    V, N = 32768, 1536
    w = to_dev(synth.q4k_matrix(V, N, 71))
    xs = [to_dev(synth.activations(1, N, seed)[0]) for seed in (72, 73, 74, 75, 76)]
    refs = [ctx.lmhead_select(w, x, V, N, 30.0) for x in xs]
    torch.cuda.synchronize()
    ex = ctx.exchange(0, 1)
    try:
        got = [ctx.lmhead_select_sharded(ex, w, x, V, N, 30.0) for x in xs]
        torch.cuda.synchronize()
        for g, ref in zip(got, refs):
            assert torch.equal(g.cand_idx, ref.cand_idx)
            assert torch.equal(g.cand_val.view(torch.int32), ref.cand_val.view(torch.int32))
            assert torch.equal(g.argmax, ref.argmax)
        ctx.check()
    finally:
        ex.close()


def test_lmhead_repeat_calls_reset_scratch(ctx):
    V, N = 4096, 256
    w = to_dev(synth.q4k_matrix(V, N, 5))
    x1 = to_dev(synth.activations(1, N, 6)[0])
    x2 = to_dev(synth.activations(1, N, 7)[0])
    a = ctx.lmhead_select(w, x1, V, N, 30.0, return_logits=True)
    b = ctx.lmhead_select(w, x2, V, N, 30.0, return_logits=True)
    c = ctx.lmhead_select(w, x1, V, N, 30.0, return_logits=True)
    assert torch.equal(a.cand_idx, c.cand_idx) and torch.equal(a.argmax, c.argmax)
    assert int(b.argmax.cpu()[0]) == int(ctx.argmax(b.logits).cpu()[0])


def test_deterministic(ctx):
    M, N = 4096, 1536
    w = to_dev(synth.q4k_matrix(M, N, 11))
    x = to_dev(synth.activations(4, N, 12))
    y1 = ctx.gemv(w, x, M, N)
    y2 = ctx.gemv(w, x, M, N)
    assert torch.equal(y1.view(torch.int32), y2.view(torch.int32))


def test_output_canaries_untouched(ctx, oracle):
    M, N, pad = 1000, 512, 64
    w = synth.q4k_matrix(M, N, 21)
    x = synth.activations(2, N, 22)
    buf = torch.full((2 * M + 2 * pad,), 12345.0, dtype=torch.float32, device=DEV)
    out = buf[pad:pad + 2 * M]
    ctx.gemv(to_dev(w), to_dev(x), M, N, out=out)
    b = buf.cpu().numpy()
    assert np.all(b[:pad] == 12345.0) and np.all(b[pad + 2 * M:] == 12345.0)
    check_gemv(oracle, b[pad:pad + 2 * M].reshape(2, M), w, x, M, N)


def test_errors_are_reported(ctx):
    w = torch.zeros(144 * 4, dtype=torch.uint8, device=DEV)
    x = torch.zeros(300, dtype=torch.float32, device=DEV)
    with pytest.raises(Q4KError, match="multiple of 256"):
        ctx.gemv(w, x, 4, 300)
    xm = torch.zeros(260, dtype=torch.float32, device=DEV)[1:257]  # 4-byte offset: misaligned
    with pytest.raises(Q4KError, match="aligned"):
        ctx.gemv(w[:144], xm, 1, 256)
    with pytest.raises(ValueError):
        ctx.gemv(w, torch.zeros(256, dtype=torch.float32, device=DEV), 8, 256)  # weight too small


def test_plan_matches_single_calls(ctx, oracle):
    from q4k import Plan

    H, I = 512, 1024
    wg = to_dev(synth.q4k_matrix(I, H, 31))
    wu = to_dev(synth.q4k_matrix(I, H, 32))
    wd_np = synth.q4k_matrix(H, I, 33)
    wd = to_dev(wd_np)
    for B in (1, 3):
        x = to_dev(synth.activations(B, H, 34))
        g = torch.empty((B, I), dtype=torch.float32, device=DEV)
        u = torch.empty_like(g)
        act = torch.empty_like(g)
        y = torch.empty((B, H), dtype=torch.float32, device=DEV)
        p = Plan(ctx, batch=B)
        p.gemv(0, wg, x, g, I, H)
        p.gemv(0, wu, x, u, I, H)
        p.gelu_mul(1, g, u, act)
        p.gemv(1, wd, act, y, H, I)
        p.commit()
        # each stage's activations fit every CTA's cache: one engine launch per stage
        assert p.launches() == 2
        p.run()
        torch.cuda.synchronize()
        g1 = ctx.gemv(wg, x, I, H)
        u1 = ctx.gemv(wu, x, I, H)
        a1 = ctx.gelu_mul(g1, u1)
        y1 = ctx.gemv(wd, a1, H, I)
        for a, b in ((g, g1), (u, u1), (act, a1), (y, y1)):
            assert torch.equal(a.view(torch.int32), b.view(torch.int32))
        check_gemv(oracle, y.cpu().numpy(), wd_np, act.cpu().numpy(), H, I)
        p.close()


@pytest.mark.parametrize("B", [1, 3, 4])
def test_plan_long_rows_split_across_warps(ctx, oracle, B):
    # a stage of rows with >= 16 super-blocks shares each 16-row tile between
    # 4 warps (one quarter of K each) and adds their sums in a fixed order:
    # two runs give the same bits, and both match the oracle
    from q4k import Plan

    M, N = 1000, 6144
    w_np = synth.q4k_matrix(M, N, 61)
    x_np = synth.activations(B, N, 62)
    w, x = to_dev(w_np), to_dev(x_np)
    y = torch.empty((B, M), dtype=torch.float32, device=DEV)
    p = Plan(ctx, batch=B)
    p.gemv(0, w, x, y, M, N)
    p.commit()
    p.run()
    torch.cuda.synchronize()
    first = y.clone()
    p.run()
    torch.cuda.synchronize()
    assert torch.equal(first.view(torch.int32), y.view(torch.int32))
    check_gemv(oracle, y.cpu().numpy(), w_np, x_np, M, N)
    p.close()


def test_plan_lmhead_matches_single_call(ctx):
    from q4k import Plan, Selection

    V, N = 8192, 768
    w = to_dev(synth.q4k_matrix(V, N, 41))
    x = to_dev(synth.activations(1, N, 42))
    ref = ctx.lmhead_select(w, x[0], V, N, 30.0, return_logits=True)
    sel = Selection(torch.empty(256, device=DEV), torch.empty(256, dtype=torch.int32, device=DEV),
                    torch.empty(1, dtype=torch.int32, device=DEV), torch.empty(V, device=DEV))
    p = Plan(ctx, batch=1)
    p.lmhead(0, w, x, V, N, 30.0, sel)
    p.commit()
    for _ in range(2):  # the scratch resets between runs
        p.run()
        torch.cuda.synchronize()
        assert torch.equal(sel.cand_idx, ref.cand_idx) and torch.equal(sel.argmax, ref.argmax)
        assert torch.equal(sel.logits.view(torch.int32), ref.logits.view(torch.int32))
    p.close()


def test_decode_step_plan_equals_serial(ctx):
    from q4k.decode import DecodeStep, E2BShape

    shape = E2BShape(layers=2, hidden=512, q=768, kv=256, ffn=1024, vocab=4096)
    step = DecodeStep(ctx, shape, batch=1)
    step.run()
    torch.cuda.synchronize()
    plan_out = {k: v.clone() for k, v in step.out.items()}
    plan_sel = (step.sel.cand_idx.clone(), step.sel.argmax.clone())
    step.run_serial()
    torch.cuda.synchronize()
    for k, v in step.out.items():
        assert torch.equal(v.view(torch.int32), plan_out[k].view(torch.int32)), k
    assert torch.equal(step.sel.cand_idx, plan_sel[0]) and torch.equal(step.sel.argmax, plan_sel[1])


def test_extreme_activation_range(ctx, oracle):
    # the hi/lo split is scaled per token by a power of two: huge and tiny x
    M, N = 64, 512
    w = synth.q4k_matrix(M, N, 51)
    for scale in (1e-20, 1e-3, 1e4, 1e12):
        x = (synth.activations(2, N, 52) * np.float32(scale)).astype(np.float32)
        y = ctx.gemv(to_dev(w), to_dev(x), M, N).cpu().numpy()
        check_gemv(oracle, y, w, x, M, N)
