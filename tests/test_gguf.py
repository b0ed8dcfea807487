"""GGUF reader (q4k/gguf.py, restating src/gguf.ts:11-101 and tensorByteSize
src/gguf.ts:383-395) against the committed fixture written by gguf-py's
GGUFWriter (tests/golden/make_gguf.py), and the tensors it loads run through
the kernels on the GPU (the weight-probe comparison of
src/diagnostics/weight-probe.ts:60-162: the device's f16 weights against the
CPU decode, bit for bit)."""
from __future__ import annotations

import struct

import numpy as np
import pytest

from q4k import gguf as G
from q4k import synth

FIXTURE = "tiny_q4k.gguf"


@pytest.fixture(scope="module")
def gf(golden_dir):
    return G.open_gguf(golden_dir / FIXTURE)


def test_header_and_metadata(gf):
    assert gf.version == 3
    kv = gf.kv
    assert kv["general.architecture"] == "gemma4"
    assert kv["gemma4.block_count"] == 1
    assert kv["gemma4.final_logit_softcapping"] == pytest.approx(30.0)
    assert kv["test.flag"] is True
    assert (kv["test.u8"], kv["test.i8"], kv["test.u16"], kv["test.i16"]) == (200, -100, 60000, -30000)
    assert kv["test.i32"] == -2_000_000_000
    assert (kv["test.u64"], kv["test.i64"]) == (2 ** 40 + 3, -(2 ** 40) - 5)
    assert kv["test.f64"] == 0.1
    assert kv["test.tokens"] == ["<pad>", "<bos>", "héllo"]
    assert kv["test.ints"] == [1, -2, 3]


def test_tensor_table_matches_gguf_py(gf, golden_dir):
    """Names, dims, types, absolute data offsets and byte sizes equal those of
    gguf-py's own reader (an independent parser of the same file)."""
    gguf = pytest.importorskip("gguf")
    r = gguf.GGUFReader(str(golden_dir / FIXTURE))
    assert gf.data_offset == r.data_offset
    assert gf.data_offset % G.ALIGNMENT == 0
    assert [t.name for t in gf.tensors] == [t.name for t in r.tensors]
    for a, b in zip(gf.tensors, r.tensors):
        assert a.dims == tuple(int(d) for d in b.shape)
        assert a.type == int(b.tensor_type)
        assert gf.data_offset + a.offset == b.data_offset
        assert a.nbytes == b.n_bytes
        assert np.array_equal(gf.tensor_bytes(a), np.asarray(b.data).reshape(-1).view(np.uint8))


def test_q4k_matrices_are_the_written_bytes(gf):
    w, M, N = gf.q4k_matrix("blk.0.attn_q.weight")
    assert (M, N) == (256, 512)
    assert np.array_equal(w, synth.q4k_matrix(256, 512, seed=11))
    e, V, NE = gf.q4k_matrix("token_embd.weight")
    assert (V, NE) == (1024, 256)
    assert np.array_equal(e, synth.q4k_matrix(1024, 256, seed=12))


def test_tensor_byte_sizes(gf):
    sizes = {t.name: t.nbytes for t in gf.tensors}
    assert sizes["blk.0.attn_norm.weight"] == 256 * 4
    assert sizes["blk.0.f16.weight"] == 256 * 2
    assert sizes["blk.0.bf16.weight"] == 64 * 2
    assert sizes["blk.0.q8_0.weight"] == 6 * 34
    assert sizes["blk.0.q5_k.weight"] == 2 * 176
    assert sizes["blk.0.q6_k.weight"] == 3 * 210
    assert sizes["blk.0.attn_q.weight"] == synth.q4k_bytes(256, 512)


def test_weight_probe_cpu(gf, oracle):
    """The oracle's f16 weights of a loaded tensor equal gguf-py's decode
    rounded to f16 (the CPU half of the weight probe)."""
    from gguf import quants
    from gguf.constants import GGMLQuantizationType

    w, M, N = gf.q4k_matrix("blk.0.attn_q.weight")
    ref = quants.dequantize(np.array(w).reshape(-1), GGMLQuantizationType.Q4_K).astype(np.float32)
    assert np.array_equal(oracle.dequant_f16(np.array(w)), ref.reshape(-1).astype(np.float16).view(np.uint16))


def test_wrong_type_rejected(gf):
    with pytest.raises(G.GGUFError, match="not Q4_K"):
        gf.q4k_matrix("blk.0.q6_k.weight")
    with pytest.raises(G.GGUFError, match="not a matrix"):
        gf.by_name["blk.0.attn_norm.weight"].matrix_shape


def test_bad_magic_and_truncation(golden_dir):
    data = bytearray((golden_dir / FIXTURE).read_bytes())
    bad = bytearray(data)
    bad[0:4] = b"GGUG"
    with pytest.raises(G.GGUFError, match="magic"):
        G.parse(bytes(bad))
    with pytest.raises(G.GGUFError, match="truncated"):
        G.parse(bytes(data[:100]))
    # a file cut inside the tensor data parses, but reading the cut tensor fails
    f = G.parse(bytes(data[:-10]))
    with pytest.raises(G.GGUFError, match="past the end"):
        f.tensor_bytes("token_embd.weight")


def test_unknown_value_and_tensor_types():
    def s(x: str) -> bytes:
        b = x.encode()
        return struct.pack("<Q", len(b)) + b

    head = struct.pack("<IIQQ", G.GGUF_MAGIC, 3, 0, 1) + s("k") + struct.pack("<I", 13)
    with pytest.raises(G.GGUFError, match="value type 13"):
        G.parse(head)
    blob = struct.pack("<IIQQ", G.GGUF_MAGIC, 3, 1, 0) + s("t") + struct.pack("<IQIQ", 1, 256, 99, 0)
    f = G.parse(blob + bytes(64))
    with pytest.raises(G.GGUFError, match="unknown tensor type 99"):
        f.tensors[0].nbytes


def test_empty_file_parses():
    f = G.parse(struct.pack("<IIQQ", G.GGUF_MAGIC, 3, 0, 0))
    assert f.tensors == [] and f.kv == {} and f.data_offset == 32


# ----------------------------------------------------------------- GPU half

@pytest.mark.gpu
def test_gguf_tensor_gemv_and_weight_probe(gf, ctx, oracle):
    torch = pytest.importorskip("torch")
    wd, M, N = G.upload_q4k(gf, "blk.0.attn_q.weight", ctx.device)
    w = np.array(gf.q4k_matrix("blk.0.attn_q.weight")[0])
    # weight probe: the device's f16 weights equal the CPU decode bit for bit
    probe = ctx.dequant_f16(wd.reshape(-1)).cpu().numpy().view(np.uint16)
    assert np.array_equal(probe, oracle.dequant_f16(w))
    # matmul through the loaded tensor, batch 1 and 3
    for B in (1, 3):
        x = synth.activations(B, N, seed=40 + B)
        y = ctx.gemv(wd, torch.from_numpy(x).to(ctx.device), M, N).cpu().numpy().reshape(B, M)
        y_ref = oracle.q4k_gemv(w, x, M, N)
        _, wn = oracle.q4k_gemv_f64(w, x, M, N)
        ok, ratio, l2 = oracle.tolerance_ok(y, y_ref, wn, x)
        assert ok, f"worst ratio {ratio:.3g}"
        assert l2 <= 1e-4


@pytest.mark.gpu
def test_gguf_tied_embedding_lm_head(gf, ctx, oracle):
    torch = pytest.importorskip("torch")
    wd, V, N = G.upload_q4k(gf, "token_embd.weight", ctx.device)
    w = np.array(gf.q4k_matrix("token_embd.weight")[0])
    cap = float(gf.kv["gemma4.final_logit_softcapping"])
    x = synth.activations(1, N, seed=77)
    sel = ctx.lmhead_select(wd, torch.from_numpy(x[0]).to(ctx.device), V, N, cap, return_logits=True)
    torch.cuda.synchronize()
    logits = oracle.logit_softcap(oracle.q4k_gemv(w, x, V, N)[0], cap)
    gl = sel.logits.cpu().numpy()
    assert np.linalg.norm(gl - logits) / np.linalg.norm(logits) <= 1e-4
    top2 = np.sort(logits)[-2:]
    if top2[1] - top2[0] > 2e-3:
        assert int(sel.argmax.cpu()[0]) == oracle.argmax(logits)
    # the fused candidates are the standalone topk256 of the device logits
    buf = ctx.topk256(sel.logits).cpu().numpy()
    assert np.array_equal(buf[1::2].view(np.uint32), sel.cand_idx.cpu().numpy().view(np.uint32))


def test_q5k_table_shape_checks(gf):
    b, vocab = gf.q5k_table("blk.0.q5_k.weight", 1)
    assert b.shape == (2, 176) and vocab == 2
    with pytest.raises(G.GGUFError):
        gf.q5k_table("blk.0.q5_k.weight", 2)  # the rows hold one layer, not two
    with pytest.raises(G.GGUFError):
        gf.q5k_table("blk.0.q6_k.weight", 1)


@pytest.mark.gpu
def test_gguf_q5k_table_through_ple_stage1(gf, ctx, oracle):
    """The Q5_K tensor of the file, used as a one-layer per-layer-embedding
    table: its decoded values (weight probe) and ple_stage1 for both rows
    equal the oracle's."""
    torch = pytest.importorskip("torch")
    b, vocab = gf.q5k_table("blk.0.q5_k.weight", 1)
    table = torch.from_numpy(np.array(b)).to(ctx.device)
    probe = ctx.q5k_dequant_f16(table.reshape(-1)).cpu().numpy().view(np.uint16)
    assert np.array_equal(probe, oracle.q5k_dequant_f16(b))
    tokens = np.array([1, 0], dtype=np.uint32)
    proj = synth.activations(2, 256, seed=78)
    nw = np.linspace(0.5, 1.5, 256).astype(np.float16).view(np.uint16)
    out = ctx.ple_stage1(table, torch.from_numpy(tokens.view(np.int32)).to(ctx.device), vocab, 1,
                         torch.from_numpy(proj).to(ctx.device), torch.from_numpy(nw.view(np.int16)).to(ctx.device),
                         1e-6).cpu().numpy()
    ref = oracle.ple_stage1(b, tokens, 1, proj, nw, 1e-6)
    # same f32 operations in the same order on both sides: at most 1 ulp apart
    ia, ib = out.view(np.int32).astype(np.int64), ref.view(np.int32).astype(np.int64)
    assert np.max(np.abs(ia - ib)) <= 1
