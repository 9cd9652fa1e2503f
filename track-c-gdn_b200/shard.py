"""Partitioning of a GDN serving step across GPUs (one process per GPU).

Decode requests and prefill sequences are independent recurrences, so the
step shards with no communication during compute:
  * decode: contiguous request blocks, each rank owning its requests' states
    (the state pool stays resident on its GPU);
  * prefill: longest-processing-time-first (LPT) bin packing of sequences by
    cost = number of 64-token chunks + a per-sequence constant (the scan's
    per-sequence setup), which bounds the makespan by 4/3 of optimal.
The step's results (decode outputs and prefill final states) end on rank 0
without a gather: each rank's kernels store them straight into rank 0's
memory (PeerResult, CUDA IPC over NVLink), and one 4-byte NCCL all-reduce
closes the step.  An NCCL gather after the compute (gather_padded) is the
fallback when the peer mapping is not possible.
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


# ---------------------------------------------------------------------------
# Results written in place across GPUs (replaces the gather)
# ---------------------------------------------------------------------------
def row_offsets(rows: Sequence[int]) -> List[int]:
    """Start row of each rank's block in a rank-major result (len world + 1)."""
    off = [0]
    for r in rows:
        if r < 0:
            raise ValueError("row counts must be >= 0")
        off.append(off[-1] + int(r))
    return off


class DeviceRows:
    """A device address handed to the destination-passing entry points
    (`decode_into`, `prefill_into`, ...), which read only `data_ptr()`."""

    def __init__(self, ptr: int):
        self._ptr = int(ptr)

    def data_ptr(self) -> int:
        return self._ptr


class CudaIpc:
    """CUDA IPC through the driver API (cuda-python): export the allocation
    that holds a pointer, map a peer's export into the current context with
    lazy peer access.  The current context must be the caller's GPU."""

    def __init__(self):
        from cuda.bindings import driver
        self._drv = driver

    def _ok(self, res, what):
        err, *vals = res
        if err != self._drv.CUresult.CUDA_SUCCESS:
            raise RuntimeError(f"{what} failed: {err}")
        return vals[0] if len(vals) == 1 else vals

    def export(self, ptr: int):
        base, _ = self._ok(self._drv.cuMemGetAddressRange(ptr), "cuMemGetAddressRange")
        handle = self._ok(self._drv.cuIpcGetMemHandle(base), "cuIpcGetMemHandle")
        return bytes(handle.reserved), ptr - int(base)

    def open(self, handle: bytes, device: int) -> int:
        dev = self._ok(self._drv.cuCtxGetDevice(), "cuCtxGetDevice")
        if int(dev) != device:
            raise RuntimeError(f"current CUDA context is on device {int(dev)}, not {device}")
        h = self._drv.CUipcMemHandle()
        h.reserved = handle
        flags = self._drv.CUipcMem_flags.CU_IPC_MEM_LAZY_ENABLE_PEER_ACCESS
        return int(self._ok(self._drv.cuIpcOpenMemHandle(h, flags), "cuIpcOpenMemHandle"))

    def close(self, ptr: int) -> None:
        self._ok((self._drv.cuIpcCloseMemHandle(ptr)[0], None), "cuIpcCloseMemHandle")


class PeerResult:
    """A step result that lives on rank `dst` and that every rank writes in
    place, so no gather runs after the step.

    `dst` allocates two rank-major buffers [sum(rows), *row_shape] (rank r's
    rows start at row_offsets(rows)[r]), one allocation, and sends its CUDA
    IPC handle to the group; every other rank maps it with lazy peer access.
    Steps alternate between the two buffers.  A rank passes `rows_for_me()`
    (this step's buffer) as the destination of its decode or prefill call,
    and the kernels' stores cross NVLink while the rest of the step still
    computes.  `publish()` closes a step: a 4-byte all-reduce on the current
    stream (NCCL), or a device sync and a barrier (other backends), then the
    next step's buffer becomes current.  Each rank joins it after its
    kernels, so once it returns on `dst`, every rank's kernels have finished
    and their stores are in `tensor()` (the buffer of the step just
    published).

    Ordering rule: the other ranks write step s+1 into the other buffer
    while `dst` still reads step s, and write step s's buffer again only in
    step s+2, after they have passed publish() of step s+1 -- which `dst`
    joins only after whatever it queued before it on the same stream.  So
    `dst` must consume step s's result (host reads, or reads queued on the
    stream that publish() runs on) before it calls publish() for step s+1.

    Only plain stores reach the peer memory (no TMA, no multicast).  Call
    `close()` on every rank before the process group goes away."""

    def __init__(self, rows: Sequence[int], row_shape: Sequence[int], dtype: torch.dtype,
                 device: torch.device, group=None, dst: int = 0, ipc=None):
        import torch.distributed as dist

        self._dist, self._group, self.dst = dist, group, dst
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if len(rows) != self.world:
            raise ValueError(f"{len(rows)} row counts for a world of {self.world}")
        self.offsets = row_offsets(rows)
        self.row_shape = tuple(int(x) for x in row_shape)
        self.dtype = dtype
        self.device = torch.device(device)
        self.row_bytes = int(np.prod(self.row_shape, dtype=np.int64)) * torch.empty(
            0, dtype=dtype).element_size()
        self._ipc = ipc if ipc is not None else CudaIpc()
        self._sync()  # the device's context exists and is current before any mapping
        self._mapped = None
        self._buf = None
        self._cur = 0       # buffer the current step writes
        self._published = None  # buffer of the last published step
        total = self.offsets[-1]
        # each buffer starts on a 256-byte boundary inside the allocation
        self._rows_pad = max(total, 1)
        per = self._rows_pad * self.row_bytes
        self._buf_bytes = (per + 255) // 256 * 256
        payload = [None]
        if self.rank == dst:
            elems = 2 * self._buf_bytes // torch.empty(0, dtype=dtype).element_size()
            self._buf = torch.empty(elems, dtype=dtype, device=self.device)
            payload = [self._ipc.export(self._buf.data_ptr())]
        dist.broadcast_object_list(payload, src=dst, group=group,
                                   device=self.device if self._nccl() else None)
        error = None
        if self.rank == dst:
            self._base = self._buf.data_ptr()
        else:
            handle, offset = payload[0]
            try:
                self._mapped = self._ipc.open(handle, self.device.index or 0)
                self._base = self._mapped + offset
            except Exception as e:  # noqa: BLE001 -- reported on every rank below
                error = f"rank {self.rank}: {e}"
        # every rank learns whether all mappings succeeded, so that all of
        # them raise (or none does) and their collectives stay in step
        self._flag = torch.zeros(1, dtype=torch.int32,
                                 device=self.device if self._nccl() else "cpu")
        self._flag.fill_(0 if error is None else 1)
        dist.all_reduce(self._flag, group=group)
        if int(self._flag.item()) != 0:
            if self._mapped is not None:
                self._ipc.close(self._mapped)
                self._mapped = None
            self._buf = None
            raise RuntimeError("peer mapping of the result buffer failed on "
                               f"{int(self._flag.item())} rank(s)" + (f" ({error})" if error else ""))
        if not self._nccl():
            self._flag = None

    def _nccl(self) -> bool:
        return self._dist.get_backend(self._group) == "nccl"

    def rows_for(self, rank: int) -> DeviceRows:
        """Where `rank`'s first row of the current step goes, as an address
        valid in this process (this rank's own block when rank == self.rank)."""
        return DeviceRows(self._base + self._cur * self._buf_bytes
                          + self.offsets[rank] * self.row_bytes)

    def rows_for_me(self) -> DeviceRows:
        return self.rows_for(self.rank)

    def publish(self, *others: "PeerResult") -> None:
        """Close the current step (collective) and make the other buffer the
        next step's.  PeerResults of the same group written in the same step
        can be passed as `others`: the one collective closes the step for
        all of them."""
        for o in others:
            if o._group is not self._group or o.dst != self.dst:
                raise ValueError("results published together must share group and dst")
        if self._flag is not None:
            self._dist.all_reduce(self._flag, group=self._group)
        else:
            self._sync()
            self._dist.barrier(group=self._group)
        for r in (self, *others):
            r._published = r._cur
            r._cur ^= 1

    def _sync(self) -> None:
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)

    def _view(self, which: int) -> torch.Tensor:
        esz = self._buf.element_size()
        start = which * self._buf_bytes // esz
        n = self.offsets[-1] * self.row_bytes // esz
        return self._buf[start:start + n].view((self.offsets[-1],) + self.row_shape)

    def tensor(self) -> torch.Tensor:
        """The whole rank-major result of the last published step (on `dst`
        only; before the first publish(), the current step's buffer)."""
        if self._buf is None:
            raise RuntimeError("the result lives on rank %d" % self.dst)
        return self._view(self._cur if self._published is None else self._published)

    def close(self) -> None:
        """Unmap (all ranks, after their last kernel), then free on `dst`."""
        self._sync()
        if self._mapped is not None:
            self._ipc.close(self._mapped)
            self._mapped = None
        if self._nccl():
            self._dist.barrier(group=self._group, device_ids=[self.device.index])
        else:
            self._dist.barrier(group=self._group)
        self._buf = None
