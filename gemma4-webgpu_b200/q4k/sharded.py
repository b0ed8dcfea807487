"""Vocabulary-parallel LM head over torch.distributed (one rank per GPU).

The reference runs its LM head on one device: the lmHead matmul over all
262144 rows, logitSoftcap, then argmax or topk256 (src/engine.ts:1686-1741).
Rows are independent and the selection reduces per residue class (index mod
256, shaders/topk256.wgsl:5-21), so the head shards by rows:

  * rank r of G owns rows [r*V/G, (r+1)*V/G); V/G is a multiple of 256, so a
    shard holds whole residue classes' slices and its candidates carry global
    indices (q4k_lmhead_select with row_offset = r*V/G);
  * one all-gather moves each rank's 256 candidates (f32 value + u32 index,
    2 KB) to every rank;
  * every rank merges the G candidate sets with q4k_merge_candidates: the
    per-residue maximum (lower index on ties) and the reference's argmax tree
    over the merged set, which equal the unsharded head's outputs.

The only collective is that 2 KB-per-rank all-gather; the weights never move.

With `fused=True` there is no collective call at all: each rank's LM-head
launch writes its candidates straight into every rank's mailbox over NVLink,
waits (bounded) for the other ranks' and merges them (q4k_exchange_* and
q4k_lmhead_select_sharded); the process group only carries the one-time
exchange of the mailboxes' IPC handles.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

from .ops import Context, Selection

SelectFn = Callable[[torch.Tensor, torch.Tensor, torch.Tensor], None]
MergeFn = Callable[[torch.Tensor, torch.Tensor], Selection]


def shard_range(V: int, world: int, rank: int) -> tuple[int, int]:
    """(first row, rows) of `rank`'s shard of a V-row head split G ways."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if V % (256 * world) != 0:
        raise ValueError(f"V={V} must be a multiple of 256*G={256 * world} (whole residue classes per shard)")
    rows = V // world
    return rank * rows, rows


class ShardedLMHead:
    """One rank's part of a G-way vocabulary-parallel LM head.

    `__call__(w_shard, x)` runs the fused head on this rank's rows, all-gathers
    the candidates and returns the merged Selection (identical on every rank).
    The default select/merge steps are the libq4k kernels on the rank's GPU;
    `select` / `merge` replace them (the CPU tests drive the partitioning and
    the collective with the oracle instead).
    """

    def __init__(self, V: int, N: int, cap: float = 30.0, ctx: Context | None = None,
                 group: dist.ProcessGroup | None = None, select: SelectFn | None = None,
                 merge: MergeFn | None = None, device: torch.device | None = None, fused: bool = False):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.V, self.N, self.cap = V, N, cap
        self.row0, self.rows = shard_range(V, self.world, self.rank)
        self.ctx = ctx
        if (select is None or merge is None) and ctx is None:
            raise ValueError("the GPU select/merge steps need a Context")
        self.device = device or (ctx.device if ctx is not None else torch.device("cpu"))
        self._select = select or self._gpu_select
        self._merge = merge or self._gpu_merge
        # send buffer: this rank's 256 values then 256 indices (bit patterns), one collective
        self.send = torch.empty(512, dtype=torch.float32, device=self.device)
        self.recv = torch.empty(self.world * 512, dtype=torch.float32, device=self.device)
        self._argmax = torch.empty(1, dtype=torch.int32, device=self.device)
        self._use_into_tensor = dist.get_backend(group) == "nccl"
        self.fused = fused
        self.ex = None
        if fused:
            if ctx is None:
                raise ValueError("the fused exchange needs a Context")
            self.ex = ctx.exchange(self.rank, self.world)
            h = torch.tensor(list(self.ex.handle), dtype=torch.uint8,
                             device=self.device if self._use_into_tensor else torch.device("cpu"))
            got = [torch.empty_like(h) for _ in range(self.world)]
            dist.all_gather(got, h, group=group)
            for p, t in enumerate(got):
                self.ex.open(p, bytes(t.cpu().tolist()))
            dist.barrier(group=group)  # every mailbox is mapped everywhere before the first call

    # the shard's candidates land in the send buffer
    def _gpu_select(self, w_shard: torch.Tensor, x: torch.Tensor, send: torch.Tensor) -> None:
        out = Selection(cand_val=send[:256], cand_idx=send[256:].view(torch.int32), argmax=self._argmax,
                        logits=None)
        self.ctx.lmhead_select(w_shard, x, self.rows, self.N, self.cap, row_offset=self.row0, out=out)

    def _gpu_merge(self, vals: torch.Tensor, idx: torch.Tensor) -> Selection:
        return self.ctx.merge_candidates(vals, idx)

    def __call__(self, w_shard: torch.Tensor, x: torch.Tensor) -> Selection:
        if self.fused:
            return self.ctx.lmhead_select_sharded(self.ex, w_shard, x, self.rows, self.N, self.cap,
                                                  row_offset=self.row0)
        self._select(w_shard, x, self.send)
        if self._use_into_tensor:
            dist.all_gather_into_tensor(self.recv, self.send, group=self.group)
        else:
            dist.all_gather(list(self.recv.view(self.world, 512).unbind(0)), self.send, group=self.group)
        g = self.recv.view(self.world, 2, 256)
        vals = g[:, 0].contiguous()
        idx = g[:, 1].contiguous().view(torch.int32)
        return self._merge(vals, idx)

    def close(self) -> None:
        if self.ex is not None:
            self.ex.close()
            self.ex = None
