"""One rank of the 2..8-GPU sharded LM-head check (launched by
tests/test_multi_gpu.py through torchrun; not collected by pytest).

Every rank builds the same seeded 262144 x 1536 head, keeps its row shard on
its GPU, runs q4k.sharded.ShardedLMHead (fused head on the shard, NCCL
all-gather of the candidates, merge; then the exchange fused into the
launch) on six different inputs back to back and compares each call's merged
candidates and argmax with the unsharded fused head run on its own GPU.  Prints one line
"rank R ok" or raises.
"""
from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "gemma4-webgpu_b200"))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from q4k import Context, synth  # noqa: E402
from q4k.sharded import ShardedLMHead  # noqa: E402


def main() -> None:
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60))
    rank = dist.get_rank()
    try:
        V, N = 262144, 1536
        ctx = Context(local)
        w = torch.from_numpy(synth.q4k_matrix(V, N, 777)).cuda()
        # a different input on every call: a merge that read a slot the
        # next call had already overwritten would show up as a mismatch
        xs = [torch.from_numpy(synth.activations(1, N, seed)[0]).cuda() for seed in range(778, 784)]
        refs = [ctx.lmhead_select(w, x, V, N, 30.0) for x in xs]
        torch.cuda.synchronize()
        for fused in (False, True):
            head = ShardedLMHead(V, N, 30.0, ctx=ctx, fused=fused)
            w_shard = w[head.row0:head.row0 + head.rows]
            # back to back, no host synchronization between calls
            merged = []
            for x in xs:
                m = head(w_shard, x)
                merged.append((m.cand_idx.clone(), m.cand_val.clone(), m.argmax.clone()))
            torch.cuda.synchronize()
            for i, ((idx, val, am), ref) in enumerate(zip(merged, refs)):
                assert torch.equal(idx, ref.cand_idx), f"call {i}: candidate indices differ (fused={fused})"
                assert torch.equal(val.view(torch.int32), ref.cand_val.view(torch.int32)), \
                    f"call {i}: values differ (fused={fused})"
                assert torch.equal(am, ref.argmax), f"call {i}: argmax differs (fused={fused})"
            ctx.check()
            dist.barrier()
            head.close()
        print(f"rank {rank} ok", flush=True)
        ctx.close()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
