"""One rank of the 2..8-GPU sharded LM-head check (launched by
tests/test_multi_gpu.py through torchrun; not collected by pytest).

Every rank builds the same seeded 262144 x 1536 head, keeps its row shard on
its GPU, runs q4k.sharded.ShardedLMHead (fused head on the shard, NCCL
all-gather of the candidates, merge) and compares the merged candidates and
argmax with the unsharded fused head run on its own GPU.  Prints one line
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
        x = torch.from_numpy(synth.activations(1, N, 778)[0]).cuda()
        ref = ctx.lmhead_select(w, x, V, N, 30.0)
        for fused in (False, True):
            head = ShardedLMHead(V, N, 30.0, ctx=ctx, fused=fused)
            for _ in range(3):  # repeated calls: scratch and mailboxes reset between calls
                merged = head(w[head.row0:head.row0 + head.rows], x)
                torch.cuda.synchronize()
                assert torch.equal(merged.cand_idx, ref.cand_idx), f"candidate indices differ (fused={fused})"
                assert torch.equal(merged.cand_val.view(torch.int32), ref.cand_val.view(torch.int32)), \
                    f"values differ (fused={fused})"
                assert torch.equal(merged.argmax, ref.argmax), f"argmax differs (fused={fused})"
            ctx.check()
            dist.barrier()
            head.close()
        print(f"rank {rank} ok", flush=True)
        ctx.close()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
