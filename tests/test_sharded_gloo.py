"""The vocabulary-parallel LM head's host logic on CPU ranks (gloo, world 2 and 4).

q4k.sharded.ShardedLMHead partitions the head's rows, all-gathers each rank's
256 candidates and merges them.  Here the per-shard selection is the oracle
(GEMV + softcap + topk256 over the shard, indices made global) and the merge
a numpy restatement of q4k_merge_candidates, so the test exercises the shard
ranges and the collective without a GPU; every rank must end with the
unsharded head's candidates and argmax.  (The merge kernel itself is checked
against the unsharded head on the GPU in test_gpu_parity.py.)
"""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

ROOT = Path(__file__).resolve().parents[1]
V, N, CAP = 4096, 512, 30.0
SEED = 4242


def _paths():
    for p in (ROOT / "gemma4-webgpu_b200", ROOT / "oracle"):
        if str(p) not in sys.path:
            sys.path.insert(0, str(p))


def _merge_np(vals: np.ndarray, idx: np.ndarray):
    """q4k_merge_candidates restated: per residue the larger value, the lower
    index on ties (NaN never wins), then the argmax tree of
    shaders/argmax.wgsl:21-27 over the merged 256 (partner wins only when
    strictly greater)."""
    G = vals.shape[0]
    out_v = vals[0].copy()
    out_i = idx[0].copy()
    for g in range(1, G):
        for r in range(256):
            v, i = vals[g, r], idx[g, r]
            if v > out_v[r] or (v == out_v[r] and i < out_i[r]):
                out_v[r], out_i[r] = v, i
    tv, ti = out_v.copy(), out_i.copy()
    st = 128
    while st > 0:
        for t in range(st):
            if tv[t + st] > tv[t]:
                tv[t], ti[t] = tv[t + st], ti[t + st]
        st //= 2
    return out_v, out_i, int(ti[0])


def planted_logits(oracle, world: int) -> np.ndarray:
    """The head's softcapped logits with injected hazards: a tie between two
    shards in one residue class (the lower global index must win), a tie for
    the global maximum between shards (the argmax tree's rule decides), and
    a NaN row (never selected)."""
    from q4k import synth

    w = synth.q4k_matrix(V, N, SEED)
    x = synth.activations(1, N, SEED + 1)
    logits = oracle.logit_softcap(oracle.q4k_gemv(w, x, V, N)[0], CAP).copy()
    last = (world - 1) * (V // world)  # first row of the last shard: same residues as shard 0
    logits[7] = logits[last + 7] = np.float32(29.5)
    logits[300] = logits[last + 300] = logits[V // world + 20] = np.float32(29.9)
    logits[123] = np.float32(np.nan)
    logits[last + 123] = np.float32(np.nan)
    return logits


def _rank_main(rank: int, world: int, port: int, results, mode: str = "gemv"):
    """One CPU rank.  mode "gemv": the shard's logits from the oracle GEMV;
    "planted": the shard of planted_logits; "fail": rank 1 raises before the
    all-gather, the others must get an error from the collective (bounded by
    the process group's timeout) instead of hanging.  Each rank records its
    outcome in `results`."""
    from datetime import timedelta

    _paths()
    import oracle as O
    from q4k import synth
    from q4k.ops import Selection
    from q4k.sharded import ShardedLMHead

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    try:
        w = synth.q4k_matrix(V, N, SEED)
        x = synth.activations(1, N, SEED + 1)
        full = planted_logits(O, world) if mode == "planted" else None

        def select(w_shard, x_t, send):
            rows = head.rows
            if mode == "fail" and rank == 1:
                raise RuntimeError("injected shard failure")
            if full is not None:
                logits = full[head.row0:head.row0 + rows]
            else:
                logits = O.logit_softcap(O.q4k_gemv(w_shard.numpy(), x_t.numpy()[None, :], rows, N)[0], CAP)
            vals, idx = O.topk256(np.ascontiguousarray(logits))
            send[:256] = torch.from_numpy(vals)
            send[256:] = torch.from_numpy((idx.astype(np.int64) + head.row0).astype(np.int32)).view(torch.float32)

        def merge(vals, idx):
            v, i, am = _merge_np(vals.numpy(), idx.numpy())
            return Selection(torch.from_numpy(v), torch.from_numpy(i.astype(np.int32)),
                             torch.tensor([am], dtype=torch.int32), None)

        head = ShardedLMHead(V, N, CAP, select=select, merge=merge)
        w_shard = torch.from_numpy(np.ascontiguousarray(w[head.row0:head.row0 + head.rows]))  # [rows, N/256*144]
        try:
            sel = head(w_shard, torch.from_numpy(x[0]))
        except Exception as e:  # noqa: BLE001 -- the outcome is the test's subject
            results[rank] = ("error", f"{type(e).__name__}: {e}")
            return
        results[rank] = ("ok", sel.cand_val.numpy().copy(), sel.cand_idx.numpy().copy(), int(sel.argmax[0]),
                         head.row0, head.rows)
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run_ranks(world: int, mode: str) -> dict:
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    mp.start_processes(_rank_main, args=(world, _free_port(), results, mode), nprocs=world, join=True,
                       start_method="spawn")
    return dict(results)


def _assert_all_equal_reference(results, world, ref_v, ref_i, ref_am):
    rows = sorted((results[r][4], results[r][5]) for r in range(world))
    assert rows == [(r * V // world, V // world) for r in range(world)]
    for r in range(world):
        status, v, i, am, _, _ = results[r]
        assert status == "ok", r
        assert np.array_equal(i.astype(np.uint32), ref_i), r
        assert np.array_equal(v.view(np.uint32), ref_v.view(np.uint32)), r
        assert am == ref_am, r


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_head_equals_unsharded_on_cpu_ranks(oracle, world):
    from q4k import synth

    results = _run_ranks(world, "gemv")
    w = synth.q4k_matrix(V, N, SEED)
    x = synth.activations(1, N, SEED + 1)
    logits = oracle.logit_softcap(oracle.q4k_gemv(w, x, V, N)[0], CAP)
    ref_v, ref_i = oracle.topk256(logits)
    _assert_all_equal_reference(results, world, ref_v, ref_i, oracle.argmax(logits))


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_head_injected_ties_and_nan(oracle, world):
    """Ties across shards (in one residue class, and for the global maximum)
    and NaN rows: the merged candidates and argmax equal the unsharded
    selection of shaders/topk256.wgsl / argmax.wgsl over the whole vector."""
    logits = planted_logits(oracle, world)
    ref_v, ref_i = oracle.topk256(logits)
    ref_am = oracle.argmax(logits)
    assert ref_i[7] == 7  # the lower index of the cross-shard tie
    assert not np.isnan(logits[ref_am])
    results = _run_ranks(world, "planted")
    _assert_all_equal_reference(results, world, ref_v, ref_i, ref_am)


def test_sharded_head_rank_failure_surfaces_as_error():
    """Rank 1 raises before the all-gather: every other rank's collective
    ends with an error (peer gone, or the process group's timeout) and none
    reports a result."""
    world = 4
    results = _run_ranks(world, "fail")
    assert results[1][0] == "error" and "injected shard failure" in results[1][1]
    for r in (0, 2, 3):
        assert results[r][0] == "error", (r, results[r][:1])


def test_shard_range_rejects_split_residue_classes():
    _paths()
    from q4k.sharded import shard_range

    assert shard_range(262144, 8, 3) == (98304, 32768)
    with pytest.raises(ValueError):
        shard_range(1000, 2, 0)
    with pytest.raises(ValueError):
        shard_range(4096, 2, 2)
