"""Partitioning of a GDN serving step across GPUs (one process per GPU).

Decode requests and prefill sequences are independent recurrences, so the
step shards with no communication during compute:
  * decode: contiguous request blocks, each rank owning its requests' states
    (the state pool stays resident on its GPU);
  * prefill: longest-processing-time-first (LPT) bin packing of sequences by
    cost = number of 64-token chunks + a per-sequence constant (the scan's
    per-sequence setup), which bounds the makespan by 4/3 of optimal.
The only collective is the final gather to rank 0 of the step's results
(decode outputs and prefill final states), over NCCL.
"""
from __future__ import annotations

import heapq
from dataclasses import dataclass
from typing import List, Sequence

import numpy as np
import torch

CHUNK = 64
SEQ_OVERHEAD_CHUNKS = 2


def seq_cost(length: int) -> int:
    return (int(length) + CHUNK - 1) // CHUNK + SEQ_OVERHEAD_CHUNKS


def lpt_partition(lengths: Sequence[int], world: int) -> List[List[int]]:
    """Assign sequence indices to `world` bins, longest first, each to the
    currently lightest bin (ties -> lowest rank).  Within a bin the indices
    are returned in ascending order, so each rank's tokens stay in the
    original relative order."""
    if world < 1:
        raise ValueError("world must be >= 1")
    order = sorted(range(len(lengths)), key=lambda i: (-seq_cost(lengths[i]), i))
    heap = [(0, r) for r in range(world)]
    bins: List[List[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        bins[r].append(i)
        heapq.heappush(heap, (load + seq_cost(lengths[i]), r))
    return [sorted(b) for b in bins]


def block_partition(n: int, world: int, rank: int) -> slice:
    """Contiguous block of n items for `rank` (sizes differ by at most one)."""
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return slice(lo, lo + base + (1 if rank < extra else 0))


@dataclass
class PrefillShard:
    seq_ids: np.ndarray          # global sequence indices owned by this rank
    token_index: np.ndarray      # global token indices, concatenated per sequence
    cu_seqlens: np.ndarray       # local int64 offsets [n_local + 1]

    @property
    def num_tokens(self) -> int:
        return int(self.cu_seqlens[-1])


def prefill_shard(cu_seqlens: np.ndarray, world: int, rank: int) -> PrefillShard:
    cu = np.asarray(cu_seqlens, dtype=np.int64)
    lengths = np.diff(cu)
    ids = np.asarray(lpt_partition(lengths.tolist(), world)[rank], dtype=np.int64)
    local_cu = np.zeros(len(ids) + 1, np.int64)
    local_cu[1:] = np.cumsum(lengths[ids])
    if len(ids):
        tok = np.concatenate([np.arange(cu[i], cu[i + 1], dtype=np.int64) for i in ids])
    else:
        tok = np.zeros(0, np.int64)
    return PrefillShard(ids, tok, local_cu)


def gather_padded(t: torch.Tensor, max_rows: int, group=None, dst: int = 0):
    """Gather a [rows, ...] tensor from every rank to `dst`, padding each
    contribution to `max_rows` rows (NCCL gathers need equal sizes).  Returns
    the stacked [world, max_rows, ...] tensor on dst and None elsewhere."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if t.shape[0] < max_rows:
        pad = torch.zeros((max_rows - t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype,
                          device=t.device)
        t = torch.cat([t, pad])
    out = None
    if rank == dst:
        out = torch.empty((world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
        dist.gather(t.contiguous(), list(out.unbind(0)), dst=dst, group=group)
    else:
        dist.gather(t.contiguous(), None, dst=dst, group=group)
    return out


def unpad_gathered(stacked: torch.Tensor, counts: Sequence[int], order: Sequence[Sequence[int]],
                   total: int) -> torch.Tensor:
    """Reassemble rows gathered with gather_padded into global order: rank r
    contributed rows for global indices order[r] (first counts[r] rows)."""
    out = torch.empty((total,) + tuple(stacked.shape[2:]), dtype=stacked.dtype,
                      device=stacked.device)
    for r, (cnt, ids) in enumerate(zip(counts, order)):
        if cnt:
            idx = torch.as_tensor(np.asarray(ids, np.int64), device=stacked.device)
            out[idx] = stacked[r, :cnt]
    return out
