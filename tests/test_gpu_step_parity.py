"""The benchmarked decode step, at its full size, against the oracle.

bench.py times config 3: 35 E2B-shaped layers x {q, k, v, o, gate, up, down}
plus the 262144-row LM head, recorded as a two-launch plan (every GEMV but
down and the fused LM head in one engine launch; gelu_mul + the 35 downs in
the second), and the same sweep at 4 activation rows (the plan plus one
q4k_select_rows launch).  These tests build that step exactly as bench.py
does (q4k.decode.DecodeStep with E2BShape()) and compare every output it
produces with the oracle -- the per-token dispatch list of
encodeTransformerPass and sampleNextTokenSubmit (src/engine.ts:1539-1619,
1686-1741):

  * every layer's q/k/v/o/gate/up/down output under the GEMV contract
    (per output 1e-3 relative + 1e-6 |w||x|, L2 relative 1e-4), down against
    the oracle fed with the step's own gelu_mul output, and the whole
    gate/up -> gelu_mul -> down chain against the oracle's chain in L2;
  * gelu_mul elementwise (CUDA tanhf vs libm: a few ulp of the tanh term);
  * the 256 per-residue candidates and the argmax exactly, except residues
    (or an argmax) whose oracle top-2 gap is inside the f32 summation noise,
    which are counted and bounded.
"""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from q4k import synth  # noqa: E402
from test_gpu_parity import L2_TOL, check_gemv  # noqa: E402

pytestmark = pytest.mark.gpu

GAP_TOL = 2e-3  # logits gap below which two candidates count as a near-tie


@pytest.fixture(scope="module")
def full_step(ctx):
    from q4k.decode import DecodeStep, E2BShape

    step = DecodeStep(ctx, E2BShape(), batch=1)
    yield step
    step._plan = None


def _host_weights(shape):
    """The step's matrices regenerated on the host from the same seeds."""
    from q4k.decode import LAYER_MATS, layer_shapes, matrix_seed

    shapes = layer_shapes(shape)
    for layer in range(shape.layers):
        yield layer, {name: synth.q4k_matrix(*shapes[name], matrix_seed(layer, name)) for name in LAYER_MATS}


def _check_layers(oracle, step):
    from q4k.decode import layer_shapes

    s = step.shape
    shapes = layer_shapes(s)
    x_h = step.x_h.cpu().numpy()
    x_attn = step.x_attn.cpu().numpy()
    worst = 0.0
    for layer, W in _host_weights(s):
        out = {name: step.out[(layer, name)].cpu().numpy() for name in shapes}
        for name in ("q", "k", "v", "o", "gate", "up"):
            M, N = shapes[name]
            worst = max(worst, check_gemv(oracle, out[name], W[name], x_attn if name == "o" else x_h, M, N))
        act = step.act[layer].cpu().numpy()
        act_ref = oracle.gelu_mul(out["gate"], out["up"])
        bound = 1e-6 * np.abs(out["gate"] * out["up"]) + 1e-6 * np.abs(act_ref)
        assert np.all(np.abs(act - act_ref) <= bound), f"layer {layer}: gelu_mul"
        M, N = shapes["down"]
        worst = max(worst, check_gemv(oracle, out["down"], W["down"], act, M, N))
        # the chain against the oracle's own chain
        g_ref = oracle.q4k_gemv(W["gate"], x_h, *shapes["gate"])
        u_ref = oracle.q4k_gemv(W["up"], x_h, *shapes["up"])
        y_ref = oracle.q4k_gemv(W["down"], oracle.gelu_mul(g_ref, u_ref), M, N)
        l2 = np.linalg.norm(out["down"] - y_ref) / np.linalg.norm(y_ref)
        assert l2 <= L2_TOL, f"layer {layer}: chained down L2 {l2:.3g}"
    return worst


def _check_selection(oracle, logits_ref, cand_val, cand_idx, argmax):
    """Candidates/argmax of one row against the oracle's logits: exact
    outside near-ties; returns the number of near-tie residues."""
    vals_ref, idx_ref = oracle.topk256(logits_ref)
    residues = np.arange(logits_ref.size) % 256
    ambiguous = 0
    for r in range(256):
        mem = logits_ref[residues == r]
        top2 = np.sort(mem)[-2:]
        if top2[1] - top2[0] <= GAP_TOL:
            ambiguous += 1
            assert logits_ref[cand_idx[r]] >= top2[1] - GAP_TOL, r
            continue
        assert cand_idx[r] == idx_ref[r], f"residue {r}: {cand_idx[r]} vs {idx_ref[r]}"
        assert abs(cand_val[r] - vals_ref[r]) <= 1e-3, (r, cand_val[r], vals_ref[r])
    top2 = np.sort(logits_ref)[-2:]
    if top2[1] - top2[0] > GAP_TOL:
        assert argmax == oracle.argmax(logits_ref)
    else:
        assert logits_ref[argmax] >= top2[1] - GAP_TOL
    return ambiguous


def _lm_head_logits(oracle, step, x):
    from q4k.decode import LMHEAD_SEED

    s = step.shape
    w = synth.q4k_matrix(s.vocab, s.hidden, LMHEAD_SEED)
    return w, np.stack([oracle.logit_softcap(oracle.q4k_gemv(w, x[b:b + 1], s.vocab, s.hidden)[0], s.softcap)
                        for b in range(x.shape[0])])


def test_full_step_batch1_matches_oracle(full_step, oracle):
    step = full_step
    assert step.plan().launches() == 2
    step.run()
    torch.cuda.synchronize()
    _check_layers(oracle, step)
    _, logits = _lm_head_logits(oracle, step, step.x_h.cpu().numpy())
    amb = _check_selection(oracle, logits[0], step.sel.cand_val.cpu().numpy(),
                           step.sel.cand_idx.cpu().numpy().view(np.uint32), int(step.sel.argmax.cpu()[0]))
    assert amb <= 8, f"{amb} near-tie residues"


def test_full_step_batch4_matches_oracle(ctx, full_step, oracle):
    from q4k.decode import DecodeStep, E2BShape

    step = DecodeStep(ctx, E2BShape(), batch=4, share_weights_with=full_step)
    step.run()
    torch.cuda.synchronize()
    _check_layers(oracle, step)
    _, logits_ref = _lm_head_logits(oracle, step, step.x_h.cpu().numpy())
    logits = step.logits.cpu().numpy()  # softcapped in place by q4k_select_rows
    for b in range(4):
        l2 = np.linalg.norm(logits[b] - logits_ref[b]) / np.linalg.norm(logits_ref[b])
        assert l2 <= L2_TOL, f"row {b}: logits L2 {l2:.3g}"
        amb = _check_selection(oracle, logits_ref[b], step.cand_val[b].cpu().numpy(),
                               step.cand_idx[b].cpu().numpy().view(np.uint32), int(step.argmax[b].cpu()))
        assert amb <= 8, f"row {b}: {amb} near-tie residues"
