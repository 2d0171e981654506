"""Multi-GPU sharding of one sentence corpus, one process per GPU.

The reference embeds its corpus on one GPU in a host loop (bench/corpus.cu:80-128: sort by
length, cut batches, one bert_embed per batch, results back to corpus order). Here every
rank holds the same corpus description, plans it with bbh_plan_batches(..., world) --
length-sorted batches assigned to ranks by longest-processing-time on their FLOPs, a
deterministic plan, so every rank computes the same one without communicating -- runs its
own batches, and the fp16 [n, 384] embeddings are gathered to rank 0 in corpus order with
one collective (NCCL over NVLink on GPUs, gloo in the CPU tests).

Host-side logic only: no kernels here.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch
import torch.distributed as dist

import bbh


@dataclass
class ShardBatch:
    plan_batch: int     # index of the batch in the plan
    row: int            # first row of the batch in this rank's plan-order output
    count: int          # sentences
    tok: int            # first token of the batch in this rank's packed ids
    tokens: int
    max_len: int
    cu: np.ndarray      # [count + 1] int32, relative to tok


@dataclass
class RankShard:
    rank: int
    order: np.ndarray   # corpus indices of this rank's sentences, plan order
    ids: np.ndarray     # packed ids of those sentences, plan order
    types: np.ndarray
    batches: list
    max_tokens: int     # largest batch (tokens)
    max_len: int


def shard(plan: "bbh.CorpusPlan", rank: int, ids: np.ndarray, types: np.ndarray, offsets: np.ndarray) -> RankShard:
    """This rank's batches of `plan` with their tokens packed back to back (vectorised)."""
    order = plan.rank_order(rank).astype(np.int64)
    lens = (offsets[order + 1] - offsets[order]).astype(np.int64)
    starts = offsets[order]
    tot = int(lens.sum())
    excl = np.zeros(lens.size, np.int64)
    if lens.size:
        excl[1:] = np.cumsum(lens)[:-1]
    tok_idx = np.repeat(starts - excl, lens) + np.arange(tot, dtype=np.int64)
    batches, row, tok, mt, ml = [], 0, 0, 0, 1
    for b, idx in plan.batches(rank):
        L = lens[row:row + idx.size]
        cu = np.zeros(idx.size + 1, np.int32)
        cu[1:] = np.cumsum(L)
        t = int(cu[-1])
        m = int(L.max()) if L.size else 1
        batches.append(ShardBatch(b, row, int(idx.size), tok, t, m, cu))
        row += int(idx.size)
        tok += t
        mt, ml = max(mt, t), max(ml, m)
    return RankShard(rank, order, ids[tok_idx], types[tok_idx], batches, max(mt, 1), ml)


def rank_counts(plan: "bbh.CorpusPlan", world: int) -> list:
    """Sentences per rank (every rank can compute every rank's count from the plan)."""
    return [int(plan.rank_order(r).size) for r in range(world)]


class Rank0Gather:
    """Gathers each rank's plan-order rows [m_r, 384] into rank 0's corpus-order [n, 384]
    tensor: one gather collective over rows padded to max_r m_r, then one index copy per
    rank on rank 0. Buffers are allocated once."""

    def __init__(self, plan: "bbh.CorpusPlan", world: int, rank: int, n: int, device, dtype=torch.float16,
                 width: int = 384):
        self.world, self.rank = world, rank
        self.counts = rank_counts(plan, world)
        self.m_max = max(max(self.counts), 1)
        self.send = torch.zeros((self.m_max, width), dtype=dtype, device=device)
        self.parts = self.index = self.out = None
        if rank == 0:
            self.parts = [torch.empty((self.m_max, width), dtype=dtype, device=device) for _ in range(world)]
            self.index = [torch.as_tensor(plan.rank_order(r).astype(np.int64), device=device) for r in range(world)]
            self.out = torch.empty((n, width), dtype=dtype, device=device)

    def __call__(self, rows: torch.Tensor):
        """rows: this rank's [m_rank, width] plan-order rows (a view of self.send avoids a copy).
        Returns rank 0's corpus-order tensor (None on other ranks)."""
        m = self.counts[self.rank]
        if rows.data_ptr() != self.send.data_ptr():
            self.send[:m].copy_(rows[:m])
        if self.world > 1:
            dist.gather(self.send, self.parts if self.rank == 0 else None, dst=0)
        elif self.rank == 0:
            self.parts[0] = self.send
        if self.rank != 0:
            return None
        for r in range(self.world):
            self.out.index_copy_(0, self.index[r], self.parts[r][:self.counts[r]])
        return self.out
