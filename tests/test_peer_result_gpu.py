"""Results written in place on another process's GPU memory (shard.PeerResult).

Two processes, on GPUs 0 and 1 when there are two (the stores then cross
NVLink), else both on cuda:0 (CUDA IPC works between processes on one
device): rank 0 owns the rank-major result buffers, rank 1 maps them, and
each rank's decode and prefill calls store their outputs and final states
straight into them, for three steps.  After each step rank 0 recomputes
both ranks' work into its own tensors and the mapped writes must equal it
bit for bit -- while rank 1 is already storing the next step into the other
of the two alternating buffers.
Rank 1's prefill is one long sequence, so its final state comes from the
segmented evaluation's TAIL items; rank 0's is a ragged single-pass batch.
The processes never wait on each other inside a kernel; the host joins them
(gloo barrier after a device synchronize).
"""
import importlib
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

DEC_ROWS = [5, 3]
PREFILL_LENS = [[100, 300, 64, 7], [4096]]
STEPS = 3


def _inputs(rank, step):
    import cases
    from gpu_util import decode_args, prefill_args
    dec = decode_args(cases.decode_inputs(seed=40 + rank + 10 * step, B=DEC_ROWS[rank]))
    pre = prefill_args(cases.prefill_inputs(seed=50 + rank + 10 * step, lens=PREFILL_LENS[rank]))
    return dec, pre


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    # rank r on GPU r when there are enough GPUs (stores cross NVLink), else
    # both ranks on GPU 0 (CUDA IPC between processes on one device)
    dev_index = rank if torch.cuda.device_count() >= world else 0
    torch.cuda.set_device(dev_index)
    dev = torch.device("cuda", dev_index)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=timedelta(seconds=120))
    try:
        gdn = importlib.import_module("track-c-gdn_b200")
        shard = importlib.import_module("track-c-gdn_b200.shard")
        dec_res = shard.PeerResult(DEC_ROWS, (1, 8, 128), torch.bfloat16, dev)
        fin_res = shard.PeerResult([len(x) for x in PREFILL_LENS], (8, 128, 128), torch.float32, dev)
        if rank == 0:  # poison both buffers; the other rank writes only after the barrier
            dec_res._buf.fill_(float("nan"))
            fin_res._buf.fill_(float("nan"))
        torch.cuda.synchronize(dev)
        dist.barrier()

        verdict = "ok"
        for step in range(STEPS):
            dec, pre = _inputs(rank, step)
            q_, k_, v_, st, A_log, a, dt, b = dec
            new_state = torch.empty_like(st)
            gdn.decode.decode_into(q_, k_, v_, st, A_log, a, dt, b, None,
                                   dec_res.rows_for_me(), new_state)
            pq, pk, pv, h0, pA, pa, pdt, pb, cu = pre
            T, N = pq.shape[0], cu.numel() - 1
            out = torch.empty(T, 8, 128, dtype=torch.bfloat16, device=dev)
            ws = gdn.prefill.alloc_workspace(T, N, dev)
            gdn.prefill.prefill_into(pq, pk, pv, h0, pA, pa, pdt, pb, cu, None, out,
                                     fin_res.rows_for_me(), ws)
            dec_res.publish(fin_res)
            if rank == 0:
                # step `step` is published; the other rank may already be
                # storing step + 1 into the other buffers while this reads
                for r in range(world):
                    (q_, k_, v_, st, A_log, a, dt, b), pre_r = _inputs(r, step)
                    o_ref, _ = gdn.decode.run(q_, k_, v_, st, A_log, a, dt, b, None)
                    _, f_ref = gdn.prefill.run(*pre_r, None)
                    lo, hi = dec_res.offsets[r], dec_res.offsets[r + 1]
                    if not torch.equal(dec_res.tensor()[lo:hi], o_ref.view(hi - lo, 1, 8, 128)):
                        verdict = f"step {step}: decode rows of rank {r} differ"
                    lo, hi = fin_res.offsets[r], fin_res.offsets[r + 1]
                    if not torch.equal(fin_res.tensor()[lo:hi], f_ref):
                        verdict = f"step {step}: final states of rank {r} differ"
        status = gdn._native.read_device_status()
        dec_res.close()
        fin_res.close()
        q.put((rank, verdict, status))
    except Exception as e:  # noqa: BLE001 -- reported to the test
        q.put((rank, f"error: {e!r}", -1))
        raise
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_peer_result_writes_equal_local_results():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
    assert res == [(0, "ok", 0), (1, "ok", 0)], res
    assert all(p.exitcode == 0 for p in procs)
