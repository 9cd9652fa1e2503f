"""Multi-GPU partitioning (host logic) and the final gather, on CPU with gloo.

The serving step shards with no collective during compute: decode requests
by contiguous blocks, prefill sequences by LPT bin packing; rank 0 gathers
the decode outputs and prefill final states at the end.
"""
import importlib
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

shard = importlib.import_module("track-c-gdn_b200.shard")


def test_block_partition_covers_everything_once():
    for n in (0, 1, 7, 4096, 4097):
        for world in (1, 2, 3, 8):
            parts = [shard.block_partition(n, world, r) for r in range(world)]
            idx = np.concatenate([np.arange(p.start, p.stop) for p in parts]) if n else np.zeros(0)
            assert np.array_equal(idx, np.arange(n))
            sizes = [p.stop - p.start for p in parts]
            assert max(sizes) - min(sizes) <= 1


def test_lpt_partition_is_a_partition_and_balanced():
    rng = np.random.default_rng(0)
    lengths = rng.integers(512, 8193, size=256).tolist()
    for world in (1, 2, 4, 8):
        bins = shard.lpt_partition(lengths, world)
        flat = sorted(i for b in bins for i in b)
        assert flat == list(range(len(lengths)))
        loads = [sum(shard.seq_cost(lengths[i]) for i in b) for b in bins]
        total = sum(shard.seq_cost(x) for x in lengths)
        # LPT is within 4/3 of optimal; with many items it is far tighter
        assert max(loads) <= total / world + max(shard.seq_cost(x) for x in lengths)
        assert max(loads) / (total / world) < 1.02


def test_lpt_partition_edge_cases():
    assert shard.lpt_partition([], 4) == [[], [], [], []]
    assert shard.lpt_partition([5], 3) == [[0], [], []]
    with pytest.raises(ValueError):
        shard.lpt_partition([1, 2], 0)


def test_prefill_shard_rebuilds_cu_seqlens():
    cu = np.array([0, 70, 70, 200, 265], np.int64)
    world = 2
    seen = []
    for r in range(world):
        s = shard.prefill_shard(cu, world, r)
        assert s.cu_seqlens[0] == 0
        lens = np.diff(s.cu_seqlens)
        assert np.array_equal(lens, np.diff(cu)[s.seq_ids])
        assert len(s.token_index) == s.num_tokens
        for k, i in enumerate(s.seq_ids):
            lo, hi = s.cu_seqlens[k], s.cu_seqlens[k + 1]
            assert np.array_equal(s.token_index[lo:hi], np.arange(cu[i], cu[i + 1]))
        seen += list(s.seq_ids)
    assert sorted(seen) == [0, 1, 2, 3]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gather_worker(rank, world, port, lengths, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        parts = shard.lpt_partition(lengths, world)
        mine = parts[rank]
        # each rank "computes" a final state per sequence: value = global seq id
        states = torch.stack([torch.full((2, 3), float(i)) for i in mine]) if mine else \
            torch.zeros(0, 2, 3)
        stacked = shard.gather_padded(states, max(len(p) for p in parts))
        if rank == 0:
            full = shard.unpad_gathered(stacked, [len(p) for p in parts], parts, len(lengths))
            q.put(full.numpy())
    finally:
        dist.destroy_process_group()


def test_gather_padded_reassembles_global_order_gloo():
    lengths = [900, 64, 5000, 17, 3000, 3000, 1]
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, world, port, lengths, q)) for r in range(world)]
    for p in procs:
        p.start()
    full = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for i in range(len(lengths)):
        assert np.all(full[i] == i)


def _failing_worker(rank, world, port, q):
    """Rank 1 dies before the gather; rank 0's gather must end with an error
    (short process-group timeout), not hang."""
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        os._exit(3)
    try:
        shard.gather_padded(torch.zeros(1, 2), 1)
        q.put("no error")
    except Exception as e:  # noqa: BLE001 -- any collective error is the expected outcome
        q.put(type(e).__name__)


def test_rank_failure_surfaces_as_error_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res != "no error"


# ---- results written in place across GPUs (PeerResult), host logic ----
def test_row_offsets():
    assert shard.row_offsets([3, 0, 5]) == [0, 3, 3, 8]
    assert shard.row_offsets([]) == [0]
    with pytest.raises(ValueError):
        shard.row_offsets([1, -1])


class _FakeIpc:
    """Stands in for CUDA IPC on CPU: the export is a fixed handle and
    offset, the mapping a fixed address; failing_rank's open raises."""
    HANDLE = bytes(range(64))
    OFFSET = 1024
    MAPPED = 1 << 40

    def __init__(self, failing_rank=None):
        self.failing_rank = failing_rank
        self.closed = []

    def export(self, ptr):
        return self.HANDLE, self.OFFSET

    def open(self, handle, device):
        assert handle == self.HANDLE
        if dist.get_rank() == self.failing_rank:
            raise OSError("mapping refused")
        return self.MAPPED

    def close(self, ptr):
        self.closed.append(ptr)


def _peer_protocol_worker(rank, world, port, failing_rank, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ipc = _FakeIpc(failing_rank)
        rows = [3, 5, 0][:world]
        try:
            res = shard.PeerResult(rows, (2, 4), torch.float32, torch.device("cpu"), ipc=ipc)
        except RuntimeError as e:
            q.put((rank, "raised", str(e)))
            return
        row_bytes = 2 * 4 * 4
        buf_bytes = (8 * row_bytes + 255) // 256 * 256  # one buffer, 256-byte rounded
        base = res.tensor().data_ptr() if rank == 0 else _FakeIpc.MAPPED + _FakeIpc.OFFSET
        ok = True
        # three steps: the destination alternates between the two buffers,
        # and dst's tensor() is the buffer of the step just published
        for step in range(3):
            mine = res.rows_for_me().data_ptr()
            ok = ok and mine == base + (step % 2) * buf_bytes + res.offsets[rank] * row_bytes
            res.publish()
            if rank == 0:
                t = res.tensor()
                ok = ok and t.data_ptr() == base + (step % 2) * buf_bytes
                ok = ok and tuple(t.shape) == (8, 2, 4)
        res.close()
        ok = ok and ipc.closed == ([] if rank == 0 else [_FakeIpc.MAPPED])
        q.put((rank, "ok" if ok else "bad addresses", None))
    finally:
        dist.destroy_process_group()


def _run_peer_protocol(world, failing_rank):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_protocol_worker, args=(r, world, port, failing_rank, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return res


def test_peer_result_addresses_and_close_gloo():
    res = _run_peer_protocol(3, None)
    assert [r[1] for r in res] == ["ok"] * 3


def test_peer_result_mapping_failure_raises_on_every_rank_gloo():
    # one rank cannot map the buffer: every rank raises, none is left waiting
    res = _run_peer_protocol(2, failing_rank=1)
    assert [r[1] for r in res] == ["raised", "raised"]
    assert all("1 rank(s)" in r[2] for r in res)
