"""q4k_lmhead_select_static, the LM head for callers that cannot allocate
device memory (no context, scratch in a fixed array inside libq4k.so).

Checked through the C ABI against q4k_lmhead_select on the same inputs, on
two calls in a row (the fixed scratch keeps the first call's contents, and
the second call must not see them).  This file sorts last so a run that stops
at the first failure has already run every other test; it also passes alone
in a fresh process, where its first call does the per-device set-up.
"""
from __future__ import annotations

import pytest

torch = pytest.importorskip("torch")

from q4k import synth  # noqa: E402
from q4k import _lib  # noqa: E402

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _run_static(L, w, x, V, N, cap):
    out_val = torch.empty(256, dtype=torch.float32, device=DEV)
    out_idx = torch.empty(256, dtype=torch.int32, device=DEV)
    out_am = torch.empty(1, dtype=torch.int32, device=DEV)
    logits = torch.empty(V, dtype=torch.float32, device=DEV)
    rc = L.q4k_lmhead_select_static(w.data_ptr(), x.data_ptr(), V, N, cap, 0, logits.data_ptr(), out_val.data_ptr(),
                                    out_idx.data_ptr(), out_am.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, rc
    torch.cuda.synchronize()
    return out_val, out_idx, out_am, logits


def test_static_lmhead_matches_context_entry_point(ctx):
    L = _lib.lib()
    V, N = 32768, 1536
    w = torch.from_numpy(synth.q4k_matrix(V, N, 901)).to(DEV)
    for call, seed in enumerate((902, 903)):  # two calls in a row, different inputs
        x = torch.from_numpy(synth.activations(1, N, seed)[0]).to(DEV)
        ref = ctx.lmhead_select(w, x, V, N, 30.0, return_logits=True)
        torch.cuda.synchronize()
        val, idx, am, logits = _run_static(L, w, x, V, N, 30.0)
        assert torch.equal(idx, ref.cand_idx), call
        assert torch.equal(am, ref.argmax), call
        # the same kernel on the same inputs: bit-identical values and logits
        # (the contract's 1e-3 tolerance is therefore met with zero error)
        assert torch.equal(val.view(torch.int32), ref.cand_val.view(torch.int32)), call
        assert torch.equal(logits.view(torch.int32), ref.logits.view(torch.int32)), call
        # no bounded wait expired in either call (read from the fixed array, no allocation)
        assert L.q4k_check_static() == 0, call


def test_static_lmhead_rejects_rows_past_its_scratch():
    L = _lib.lib()
    N = 16384 + 256
    w = torch.zeros(144 * (N // 256), dtype=torch.uint8, device=DEV)
    x = torch.zeros(N, dtype=torch.float32, device=DEV)
    o = torch.zeros(256, dtype=torch.int32, device=DEV)
    rc = L.q4k_lmhead_select_static(w.data_ptr(), x.data_ptr(), 1, N, 30.0, 0, None, o.data_ptr(), o.data_ptr(),
                                    o.data_ptr(), None)
    assert rc == _lib.Q4K_ERR_SCRATCH_LIMIT
