"""The chained decode step (q4k_chain_*) against the oracle.

Each layer reads the previous layer's output through the reference's
elementwise passes (rms_norm.wgsl, fused_norm_add.wgsl,
per_head_rms_norm_no_weight.wgsl, attention at position 0, gelu_mul.wgsl;
norm weights 1), as encodeTransformerPass chains them
(src/engine.ts:1538-1626).  Checked two ways:

  * layer by layer, each GEMV against the oracle fed with the step's own
    stored input vector (recomputed in numpy from the stored residuals and
    outputs), under the GEMV contract (per output 1e-3 relative + 1e-6
    |w||x|, L2 relative 1e-4), and each stored elementwise result against
    its numpy restatement;
  * end to end, against a chain computed by the oracle alone from the same
    first input: every layer's outputs and the final norm within L2 1e-4,
    and the LM head's candidates exactly outside near-ties.
"""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from q4k import synth  # noqa: E402
from test_gpu_parity import L2_TOL, check_gemv  # noqa: E402
from test_gpu_step_parity import _check_selection  # noqa: E402

pytestmark = pytest.mark.gpu

EPS = 1e-6


def rms_norm(x: np.ndarray) -> np.ndarray:
    """rms_norm.wgsl with weight 1: x / sqrt(sum(x^2)/n + eps), in f32."""
    x = np.asarray(x, dtype=np.float32)
    ss = np.sum(x * x, dtype=np.float32)
    rms = np.float32(np.sqrt(np.float32(ss / np.float32(x.size) + np.float32(EPS))))
    return (x / rms).astype(np.float32)


def close(a, b, what):
    scale = float(np.max(np.abs(b))) or 1.0
    err = float(np.max(np.abs(a - b)))
    assert err <= 1e-5 * scale, f"{what}: max error {err:.3g} vs scale {scale:.3g}"


def _weights(shape, layers):
    from q4k.decode import LAYER_MATS, layer_shapes, matrix_seed

    shapes = layer_shapes(shape)
    return [{n: synth.q4k_matrix(*shapes[n], matrix_seed(layer, n)) for n in LAYER_MATS} for layer in range(layers)]


def _build(ctx, shape, layers=None):
    from q4k.decode import ChainedStep, DecodeStep

    step = DecodeStep(ctx, shape, batch=1)
    chain = ChainedStep(step, layers=layers)
    return step, chain


@pytest.mark.parametrize("dims", [
    dict(layers=4, hidden=1536, q=2048, kv=256, ffn=6144, vocab=16384),  # E2B-shaped, 4 layers
    dict(layers=3, hidden=512, q=1024, kv=256, ffn=1024, vocab=4096),    # other K splits
])
def test_chain_layer_by_layer(ctx, oracle, dims):
    from q4k.decode import E2BShape, layer_shapes

    shape = E2BShape(**dims)
    step, chain = _build(ctx, shape)
    assert chain.launches() == 2
    chain.run()
    torch.cuda.synchronize()
    ctx.check()
    shapes = layer_shapes(shape)
    W = _weights(shape, shape.layers)
    h = chain.h_in.cpu().numpy()
    heads = shape.q // shape.kv
    for layer in range(shape.layers):
        out = {n: t.cpu().numpy() for n, t in chain.out[layer].items()}
        n1 = rms_norm(h)
        for name in ("q", "k", "v"):
            check_gemv(oracle, out[name][None], W[layer][name], n1[None], *shapes[name])
        a = np.tile(rms_norm(out["v"]), heads)
        check_gemv(oracle, out["o"][None], W[layer]["o"], a[None], *shapes["o"])
        close(out["h_attn"], h + rms_norm(out["o"]), f"layer {layer} h_attn")
        n2 = rms_norm(out["h_attn"])
        for name, key in (("gate", "g"), ("up", "u")):
            check_gemv(oracle, out[key][None], W[layer][name], n2[None], *shapes[name])
        act_ref = oracle.gelu_mul(out["g"], out["u"])
        bound = 1e-6 * np.abs(out["g"] * out["u"]) + 1e-6 * np.abs(act_ref)
        assert np.all(np.abs(out["act"] - act_ref) <= bound), f"layer {layer} gelu_mul"
        check_gemv(oracle, out["d"][None], W[layer]["down"], out["act"][None], *shapes["down"])
        close(out["h_out"], out["h_attn"] + rms_norm(out["d"]), f"layer {layer} h_out")
        h = out["h_out"]
    close(chain.normed.cpu().numpy(), rms_norm(h), "final norm")
    # the LM head on the step's own final norm
    from q4k.decode import LMHEAD_SEED

    wl = synth.q4k_matrix(shape.vocab, shape.hidden, LMHEAD_SEED)
    logits = oracle.logit_softcap(oracle.q4k_gemv(wl, chain.normed.cpu().numpy()[None], shape.vocab,
                                                  shape.hidden)[0], shape.softcap)
    _check_chained_selection(oracle, logits, chain)
    chain.close()


def _check_chained_selection(oracle, logits, chain):
    """The chained step's candidates and argmax against the oracle's logits.
    The synthetic weights have a positive mean, so the chained residual
    stream drifts to a large common mode and most logits sit at the softcap
    (30.0 exactly in f32): those residues are exact ties whose winner depends
    on which near-threshold logits round to the cap.  Every residue's pick
    must carry its residue's maximum (within the near-tie gap) and be exact
    wherever the maximum is clear."""
    _check_selection(oracle, logits, chain.sel.cand_val.cpu().numpy(),
                     chain.sel.cand_idx.cpu().numpy().view(np.uint32), int(chain.sel.argmax.cpu()[0]))


def test_chain_end_to_end_and_repeatable(ctx, oracle):
    """Four E2B-shaped layers against a chain run by the oracle alone from
    the same input; two runs give the same bits (the stage counters reset
    themselves between runs)."""
    from q4k.decode import LMHEAD_SEED, E2BShape, layer_shapes

    shape = E2BShape(layers=4, vocab=16384)
    step, chain = _build(ctx, shape)
    chain.run()
    torch.cuda.synchronize()
    first = {k: v.clone() for k, v in chain.out[-1].items()}
    first_sel = chain.results.clone()
    chain.run()
    torch.cuda.synchronize()
    ctx.check()
    for k, v in chain.out[-1].items():
        assert torch.equal(v.view(torch.int32), first[k].view(torch.int32)), k
    assert torch.equal(chain.results, first_sel)

    shapes = layer_shapes(shape)
    W = _weights(shape, shape.layers)
    h = chain.h_in.cpu().numpy()
    heads = shape.q // shape.kv
    for layer in range(shape.layers):
        n1 = rms_norm(h)
        q, k, v = (oracle.q4k_gemv(W[layer][n], n1[None], *shapes[n])[0] for n in ("q", "k", "v"))
        o = oracle.q4k_gemv(W[layer]["o"], np.tile(rms_norm(v), heads)[None], *shapes["o"])[0]
        h_attn = h + rms_norm(o)
        n2 = rms_norm(h_attn)
        g = oracle.q4k_gemv(W[layer]["gate"], n2[None], *shapes["gate"])[0]
        u = oracle.q4k_gemv(W[layer]["up"], n2[None], *shapes["up"])[0]
        d = oracle.q4k_gemv(W[layer]["down"], oracle.gelu_mul(g, u)[None], *shapes["down"])[0]
        h = h_attn + rms_norm(d)
        got = {n: t.cpu().numpy() for n, t in chain.out[layer].items()}
        for name, ref in (("q", q), ("v", v), ("o", o), ("g", g), ("d", d), ("h_out", h)):
            l2 = np.linalg.norm(got[name] - ref) / np.linalg.norm(ref)
            assert l2 <= L2_TOL, f"layer {layer} {name}: L2 {l2:.3g}"
    normed = rms_norm(h)
    l2 = np.linalg.norm(chain.normed.cpu().numpy() - normed) / np.linalg.norm(normed)
    assert l2 <= L2_TOL
    wl = synth.q4k_matrix(shape.vocab, shape.hidden, LMHEAD_SEED)
    logits = oracle.logit_softcap(oracle.q4k_gemv(wl, normed[None], shape.vocab, shape.hidden)[0], shape.softcap)
    _check_chained_selection(oracle, logits, chain)
    chain.close()


def test_chain_rejects_bad_shapes(ctx):
    from q4k import Q4KError
    from q4k.decode import E2BShape

    # q rows of 9 super-blocks do not split into whole two-block copy stages
    with pytest.raises(Q4KError, match="super-blocks"):
        _build(ctx, E2BShape(layers=1, hidden=1536, q=2304, kv=256, ffn=6144, vocab=1024))
