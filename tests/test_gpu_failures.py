"""Failure detection on the GPU without a GPU fault.

The reference's only failure signal is device loss: `deviceLost` is set by
the device's lost promise and checked before public calls
(src/engine.ts:105, 385-388, 1677).  Here every wait inside a kernel has an
iteration limit; on expiry the kernel records it in the context's status
word, lets its copies in flight land and returns, and q4k_check reports
Q4K_ERR_TIMEOUT.  These tests make a wait run out on purpose -- a peer flag
that nothing ever sets -- with a short, caller-chosen limit, and check that
the status surfaces, clears, and leaves the context usable.
"""
from __future__ import annotations

import pytest

torch = pytest.importorskip("torch")

from q4k import Q4KError, synth  # noqa: E402
from q4k import _lib  # noqa: E402

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
SHORT_WAIT = 1 << 16  # polls: milliseconds, far above any copy's latency


def test_missing_peer_rank_times_out_and_context_recovers(ctx):
    """A two-rank sharded LM head whose rank 1 never runs: rank 0's launch
    stores its candidates, waits for rank 1's flag (never raised) until the
    short limit, records the expiry and returns.  q4k_check then reports
    Q4K_ERR_TIMEOUT once, and the next ordinary call is correct."""
    V, N = 16384, 1536
    w = torch.from_numpy(synth.q4k_matrix(V, N, 611)).to(DEV)
    x = torch.from_numpy(synth.activations(1, N, 612)[0]).to(DEV)
    ref = ctx.lmhead_select(w, x, V, N, 30.0)
    ctx.check()
    ex0, ex1 = ctx.exchange(0, 2), ctx.exchange(1, 2)
    try:
        ex0.open_local(1, ex1)  # rank 1's mailbox exists, but rank 1 never launches
        ctx.set_wait_limit(SHORT_WAIT)
        ctx.lmhead_select_sharded(ex0, w[: (V // 2) * 6 * 144], x, V // 2, N, 30.0, row_offset=0)
        with pytest.raises(Q4KError) as err:
            ctx.check()
        assert err.value.code == _lib.Q4K_ERR_TIMEOUT
        ctx.check()  # the record was cleared by the first check
    finally:
        ctx.set_wait_limit(0)
        ex0.close()
        ex1.close()
    again = ctx.lmhead_select(w, x, V, N, 30.0)
    ctx.check()
    assert torch.equal(again.cand_idx, ref.cand_idx)
    assert torch.equal(again.cand_val.view(torch.int32), ref.cand_val.view(torch.int32))
    assert torch.equal(again.argmax, ref.argmax)


def test_wait_limit_does_not_disturb_normal_calls(ctx):
    """With the short limit, calls whose waits all complete are unaffected:
    a GEMV (engine, K-split) and a batched GEMM give the default's bits."""
    M, N = 3000, 6144
    w = torch.from_numpy(synth.q4k_matrix(M, N, 621)).to(DEV)
    x = torch.from_numpy(synth.activations(64, N, 622)).to(DEV)
    y1 = ctx.gemv(w, x[:1], M, N)
    g1 = ctx.gemm(w, x, M, N)
    ctx.check()
    ctx.set_wait_limit(SHORT_WAIT)
    try:
        y2 = ctx.gemv(w, x[:1], M, N)
        g2 = ctx.gemm(w, x, M, N)
        ctx.check()
    finally:
        ctx.set_wait_limit(0)
    assert torch.equal(y1.view(torch.int32), y2.view(torch.int32))
    assert torch.equal(g1.view(torch.int32), g2.view(torch.int32))
