"""Benchmark of the B200 GDN kernel pair (qk4_v8_d128_k_last).

Default workload (benchmark config 4, "mixed serving load"): one serving step
= a decode step for 4096 requests (state updated in place, resident in HBM)
plus a ragged prefill of 256 new sequences with lengths ~U{512..8192}
(~1.1M tokens, zero initial state).  When N > 1 the decode outputs and
prefill final states end the step on rank 0: each rank's kernels store them
into rank 0's memory over NVLink (default, `--gather peer`), or an NCCL
gather runs after the compute (`--gather nccl`).  The work is a
fixed total sharded across the N ranks (decode: request blocks; prefill: LPT
bin packing by sequence), so scaling is "strong".  All inputs are seeded
synthetic tensors with the benchmark configs' value distributions.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference|triton]
                    [--workload c4|c2|c3|decode|mtp|decode_bf16]

Prints one JSON line (rank 0).  `value` is whole-job tokens/s (decode tokens
+ prefill tokens) over the device time of K steps (max over ranks);
`e2e` is the same metric through the public entry points with pinned host
inputs and outputs copied inside the timed region.  `--impl reference` times
the CPU oracle (the reference recurrence restated in C, all host threads) on
bounded samples of the same workload.  `--impl triton` times the reference's
own Triton kernels (staged unmodified under baseline/_ref) on one GPU with
the same inputs, and reports our outputs' distance from theirs.
"""
from __future__ import annotations

import argparse
import importlib
import json
import math
import os
import subprocess
import sys
import time
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

# The JSON line goes out on the original stdout; everything else that writes
# to file descriptor 1 (library banners such as NCCL's version line) is sent
# to stderr once main() has run, so stdout carries exactly one JSON line.
_JSON_FD = None


def emit(obj) -> None:
    line = (json.dumps(obj) + "\n").encode()
    if _JSON_FD is None:
        sys.stdout.write(line.decode())
        sys.stdout.flush()
    else:
        os.write(_JSON_FD, line)

HQK, HV, D = 4, 8, 128
DECODE_STATE_BYTES = HV * D * D * 4 * 2           # fp32 state read + written per request
DECODE_VEC_BYTES = 2 * HQK * D * 2 + 2 * HV * D * 2 + 2 * HV * 2  # q,k,v,out,a,b
PREFILL_FLOP_PER_TOKEN = 1_441_792                # 8 v-heads x 180,224
PREFILL_BYTES_PER_TOKEN = 6176
# backward per token: the recompute (counted as one forward) plus, per v-head
# and 64-token chunk, 4,194,304 MACs in the reverse scan (Z, dX, dS) and
# 6,815,744 in the chunk kernel (QK^T, KK^T, dO delta^T, dX delta^T, dO S_0,
# dX S_0, delta dS_C, Mq K, Mq^T Q, Msym K): 8 x 2 x 11,010,048 / 64 per token
BWD_FLOP_PER_TOKEN = PREFILL_FLOP_PER_TOKEN + 2_752_512
STATE_BYTES = HV * D * D * 4

WORKLOADS = {
    "c4": dict(desc="C4 mixed serving: decode B=4096 (in place) + ragged prefill of 256 "
                    "sequences, lengths U{512..8192}, zero initial state",
               decode_batch=4096, prefill="c4"),
    "c2": dict(desc="C2 prefill: one packed sequence T=4096, zero initial state",
               decode_batch=0, prefill="c2"),
    "c3": dict(desc="C3 ragged prefill: 32 sequences U{17..3000}, initial states randn*0.02",
               decode_batch=0, prefill="c3"),
    "decode": dict(desc="C1 decode sweep point: batch 1024, state updated in place",
                   decode_batch=1024, prefill=None),
    "mtp": dict(desc="multi-token decode (speculative verify): batch 1024 x 4 tokens per request, "
                     "state updated in place",
                decode_batch=1024, decode_tokens=4, prefill=None),
    "decode_bf16": dict(desc="decode batch 1024 with the state stored in bf16 (opt-in format), "
                             "updated in place",
                        decode_batch=1024, prefill=None, state_bf16=True),
    # profiling subset (not a bench line): the first 64 sequences of C4's
    # length list, prefill only -- inputs above L2 but a few GB on the device,
    # small enough for multi-pass ncu captures of one kernel
    "c4_64": dict(desc="profiling subset: prefill of the first 64 sequences of the C4 length list, "
                       "zero initial state", decode_batch=0, prefill="c4_64"),
    # training: one prefill backward over the C3 / C4 prefill shapes
    "bwd_c3": dict(desc="prefill backward over C3 (32 sequences U{17..3000}, initial states "
                        "randn*0.02, d_out and d_final_state random)",
                   decode_batch=0, prefill="c3", backward=True),
    "bwd_c4": dict(desc="prefill backward over the C4 prefill (256 sequences U{512..8192}, zero "
                        "initial state, d_out random, no final-state gradient)",
                   decode_batch=0, prefill="c4", backward=True),
}


def prefill_lengths(kind: str) -> np.ndarray:
    if kind == "c4":
        return np.random.default_rng(4).integers(512, 8193, size=256)
    if kind == "c4_64":
        return np.random.default_rng(4).integers(512, 8193, size=256)[:64]
    if kind == "c3":
        return np.random.default_rng(3).integers(17, 3001, size=32)
    if kind == "c2":
        return np.array([4096])
    raise ValueError(kind)


def workload_config(workload: str, world: int) -> dict:
    """The `config` of a bench line: the workload alone, so that every arm
    (b200, reference, triton) prints the identical dict for the same
    workload and N.  How an arm executes it goes under `execution`."""
    wl = WORKLOADS[workload]
    lengths = prefill_lengths(wl["prefill"]) if wl["prefill"] else np.zeros(0, np.int64)
    tokens = wl["decode_batch"] * wl.get("decode_tokens", 1) + int(lengths.sum())
    return {
        "workload": wl["desc"],
        "decode_batch": wl["decode_batch"],
        "decode_tokens_per_request": wl.get("decode_tokens", 1),
        "state_dtype": "bf16" if wl.get("state_bf16") else "fp32",
        "prefill_sequences": len(lengths),
        "prefill_tokens": int(lengths.sum()),
        "l2": ("inputs larger than L2 (no flush needed)" if tokens > 20000 else
               "inputs smaller than L2 (no flush)"),
        "parallelism": (f"shard{world}: decode request blocks, prefill LPT by sequence"
                        if world > 1 else "one GPU"),
    }


# Algorithmic work of one prefill call split between its two main kernels.
# Per 64-token chunk and v-head the path does 5 (2 C^2 D) + 3 (2 C D^2) FLOP:
# KK^T, QK^T and the W-side product (3 x 2 C^2 D) depend only on the chunk and
# are the preparation kernel's; U, P v_new and the three state products W S^T,
# K^T v_new, Q S^T (2 x 2 C^2 D + 3 x 2 C D^2) need the state and are the
# scan's.  Bytes: the preparation reads q, k, a, b; the scan reads q, k, v
# and writes the output, plus the initial / final states.
PREP_FLOP_PER_TOKEN = 8 * 3 * 2 * 64 * 64 * 128 // 64          # 393,216
SCAN_FLOP_PER_TOKEN = PREFILL_FLOP_PER_TOKEN - PREP_FLOP_PER_TOKEN  # 1,048,576
PREP_BYTES_PER_TOKEN = 2 * HQK * D * 2 + 2 * HV * 2                # 2,080
SCAN_BYTES_PER_TOKEN = 2 * HQK * D * 2 + 2 * HV * D * 2            # 6,144


def roofline_entry(kernel: str, flop: float, nbytes: float, seconds: float, peaks: dict,
                   traffic=None, sustained: bool = False) -> dict:
    """Roofline position of one timed kernel (or call): the bound is whichever
    of FLOP / tensor peak and bytes / HBM peak is longer; achieved and peak
    are in that bound's unit, so frac = max(t_tensor, t_hbm) / measured."""
    tc_peak = peaks["bf16_tflops_sustained"] if sustained else peaks["bf16_tflops"]
    t_tc = flop / (tc_peak * 1e12)
    t_hbm = nbytes / (peaks["hbm_gbs"] * 1e9)
    if t_tc >= t_hbm:
        bound, achieved, peak, unit = "tensor", flop / seconds / 1e12, tc_peak, "TFLOP/s"
        src = "bf16 sustained" if sustained else "bf16 burst"
    else:
        bound, achieved, peak, unit = "hbm", nbytes / seconds / 1e9, peaks["hbm_gbs"], "GB/s"
        src = "hbm copy"
    return {"kernel": kernel, "bound": bound, "achieved": achieved, "peak": peak, "unit": unit,
            "frac": max(t_tc, t_hbm) / seconds, "traffic": traffic,
            "algorithmic_flop": flop, "algorithmic_bytes": nbytes,
            "t_tensor_ms": t_tc * 1e3, "t_hbm_ms": t_hbm * 1e3, "measured_ms": seconds * 1e3,
            "peak_source": f"{peaks['source']} {src}"}


# ---------------------------------------------------------------------------
# measured peaks
# ---------------------------------------------------------------------------
def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return dict(hbm_gbs=d["hbm_gbs"], bf16_tflops=d["bf16_tflops"],
                    bf16_tflops_sustained=d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                    source="measured")
    return dict(hbm_gbs=6650.0, bf16_tflops=1590.0, bf16_tflops_sustained=1400.0, source="fallback")


def load_traffic(workload: str):
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return {}
    return json.loads(p.read_text()).get(workload, {})


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    """Samples this process's GPU SM clock and clock-event reasons during the
    timed region.  NVML (read-only queries) polled from a thread every 5 ms,
    so a timed region of ~100 ms still yields ~20 samples; `nvidia-smi -lms`
    is the fallback when NVML cannot be opened."""
    REASONS = (("nvmlClocksEventReasonHwSlowdown", "hw_slowdown"),
               ("nvmlClocksEventReasonHwThermalSlowdown", "hw_thermal_slowdown"),
               ("nvmlClocksEventReasonSwThermalSlowdown", "sw_thermal_slowdown"),
               ("nvmlClocksEventReasonSwPowerCap", "sw_power_cap"),
               ("nvmlClocksEventReasonHwPowerBrakeSlowdown", "hw_power_brake_slowdown"),
               ("nvmlClocksEventReasonApplicationsClocksSetting", "applications_clocks_setting"))
    SMI_FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
                  "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                  "clocks_event_reasons.sw_power_cap")

    def __init__(self, enabled: bool, device_index: int = 0):
        import threading
        self.samples = []          # (sm_mhz, frozenset(reasons))
        self.sm_max = None
        self.thread = None
        self.proc = None
        self.stop_evt = threading.Event()
        if not enabled:
            return
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            try:
                nvml_idx = torch.cuda._get_nvml_device_index(device_index)
            except Exception:  # noqa: BLE001 -- fall back to the CUDA ordinal
                nvml_idx = device_index
            self.nvml = pynvml
            self.handle = pynvml.nvmlDeviceGetHandleByIndex(nvml_idx)
            self.sm_max = float(pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM))
            self.masks = [(getattr(pynvml, a), n) for a, n in self.REASONS if hasattr(pynvml, a)]
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
        except Exception:  # noqa: BLE001 -- NVML unavailable: use nvidia-smi
            self._start_smi(device_index)

    def _poll(self):
        nv = self.nvml
        while not self.stop_evt.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)
                bits = nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                self.samples.append((float(sm), frozenset(n for m, n in self.masks if bits & m)))
            except Exception:  # noqa: BLE001 -- a failed query drops one sample
                pass
            self.stop_evt.wait(0.005)

    def _start_smi(self, device_index):
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"gdn_clocks_{os.getpid()}.csv"
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={device_index}", f"--query-gpu={self.SMI_FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"], stdout=self.fh,
                stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def _stop_smi(self):
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            try:
                sm, smax = float(parts[0]), float(parts[1])
            except (ValueError, IndexError):
                continue
            self.sm_max = smax
            self.samples.append((sm, frozenset(n for i, n in enumerate(names)
                                               if len(parts) > 2 + i and parts[2 + i].lower() == "active")))
        self.path.unlink(missing_ok=True)

    def stop(self):
        if self.thread is not None:
            self.stop_evt.set()
            self.thread.join(timeout=5)
            try:
                self.nvml.nvmlShutdown()
            except Exception:  # noqa: BLE001
                pass
            source = "nvml 5 ms"
        elif self.proc is not None:
            self._stop_smi()
            source = "nvidia-smi 50 ms"
        else:
            return None
        if not self.samples:
            return None
        sm = [x for x, _ in self.samples]
        reasons = sorted(set().union(*[r for _, r in self.samples]))
        return {"sm_mhz": float(np.median(sm)), "sm_min_mhz": min(sm), "sm_max_mhz": self.sm_max,
                "reasons": reasons, "samples": len(sm), "source": source}


def merge_clocks(dist, world, mine):
    """Clock summary over all ranks' GPUs (every rank calls this once, in the
    same place, after the timed region)."""
    if world == 1:
        return mine
    allc = [None] * world
    dist.all_gather_object(allc, mine)
    got = [c for c in allc if c]
    if not got:
        return None
    return {"sm_mhz": float(np.median([c["sm_mhz"] for c in got])),
            "sm_min_mhz": min(c["sm_min_mhz"] for c in got),
            "sm_max_mhz": max(c["sm_max_mhz"] or 0 for c in got),
            "reasons": sorted(set().union(*[c["reasons"] for c in got])),
            "samples": sum(c["samples"] for c in got), "source": got[0]["source"],
            "per_rank_sm_mhz": [c["sm_mhz"] if c else None for c in allc]}


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def make_prefill_inputs(torch, lengths, with_state, seed, dev):
    import torch.nn.functional as F
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    T = int(lengths.sum())
    N = len(lengths)
    cu = np.zeros(N + 1, np.int64)
    cu[1:] = np.cumsum(lengths)
    q = F.normalize(torch.randn(T, HQK, D, generator=g, device=dev), dim=-1).bfloat16()
    k = F.normalize(torch.randn(T, HQK, D, generator=g, device=dev), dim=-1).bfloat16()
    v = torch.randn(T, HV, D, generator=g, device=dev).bfloat16()
    a = torch.randn(T, HV, generator=g, device=dev).bfloat16()
    b = torch.randn(T, HV, generator=g, device=dev).bfloat16()
    h0 = (torch.randn(N, HV, D, D, generator=g, device=dev) * 0.02) if with_state else None
    return dict(q=q, k=k, v=v, a=a, b=b, h0=h0, cu=torch.from_numpy(cu).to(dev), T=T, N=N)


def make_decode_inputs(torch, B, seed, dev, T=1, state_bf16=False):
    import torch.nn.functional as F
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    q = F.normalize(torch.randn(B, T, HQK, D, generator=g, device=dev), dim=-1).bfloat16()
    k = F.normalize(torch.randn(B, T, HQK, D, generator=g, device=dev), dim=-1).bfloat16()
    v = torch.randn(B, T, HV, D, generator=g, device=dev).bfloat16()
    a = torch.randn(B, T, HV, generator=g, device=dev).bfloat16()
    b = torch.randn(B, T, HV, generator=g, device=dev).bfloat16()
    state = torch.randn(B, HV, D, D, generator=g, device=dev) * 0.02
    if state_bf16:
        state = state.bfloat16()
    return dict(q=q, k=k, v=v, a=a, b=b, state=state, B=B, T=T, bf16=state_bf16)


def run_decode(gdn, dec, A_log, dt_bias, out):
    """One decode step of the workload (multi-token when T > 1, bf16 state
    when the workload says so), state in place."""
    if dec.get("bf16"):
        gdn.decode.decode_bf16_state_into(dec["q"], dec["k"], dec["v"], dec["state"], A_log,
                                          dec["a"], dt_bias, dec["b"], None, out)
    elif dec["T"] == 1:
        gdn.decode.decode_into(dec["q"], dec["k"], dec["v"], dec["state"], A_log, dec["a"],
                               dt_bias, dec["b"], None, out, dec["state"])
    else:
        gdn.decode.decode_mtp_into(dec["q"], dec["k"], dec["v"], dec["state"], A_log, dec["a"],
                                   dt_bias, dec["b"], None, out, dec["state"])


def gpu_arm(args):
    import torch
    import torch.distributed as dist

    gdn = importlib.import_module("track-c-gdn_b200")
    from importlib import import_module
    shard = import_module("track-c-gdn_b200.shard")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        # NCCL would print its version banner on stdout ahead of the JSON line
        os.environ.setdefault("NCCL_DEBUG", "WARN")
        dist.init_process_group("nccl", timeout=timedelta(seconds=180),
                                device_id=dev)
    wl = WORKLOADS[args.workload]
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    A_log = (torch.rand(HV, generator=gen, device=dev) * 2.7).float()
    dt_bias = (torch.randn(HV, generator=gen, device=dev) * 0.1).float()
    if world > 1:  # same gate parameters on every rank (one model)
        dist.broadcast(A_log, 0)
        dist.broadcast(dt_bias, 0)

    # ---- this rank's shard of the workload ----
    B_total = wl["decode_batch"]
    dec_slice = shard.block_partition(B_total, world, rank)
    B = dec_slice.stop - dec_slice.start
    Tdec = wl.get("decode_tokens", 1)
    dec = (make_decode_inputs(torch, B, 100 + rank, dev, Tdec, wl.get("state_bf16", False))
           if B > 0 else None)
    pre = None
    total_prefill_tokens = 0
    seq_counts = [0] * world
    if wl["prefill"]:
        lengths = prefill_lengths(wl["prefill"])
        total_prefill_tokens = int(lengths.sum())
        parts = shard.lpt_partition(lengths.tolist(), world)
        seq_counts = [len(p) for p in parts]
        my_lengths = lengths[parts[rank]]
        pre = make_prefill_inputs(torch, my_lengths, wl["prefill"] == "c3", 200 + rank, dev)
        pre["out"] = torch.empty(pre["T"], HV, D, dtype=torch.bfloat16, device=dev)
        pre["final"] = torch.empty(pre["N"], HV, D, D, dtype=torch.float32, device=dev)
        pre["ws"] = gdn.prefill.alloc_workspace(pre["T"], pre["N"], dev)
    dec_out = torch.empty(B, Tdec, HV, D, dtype=torch.bfloat16, device=dev) if B > 0 else None
    max_seqs = max(seq_counts) if seq_counts else 0
    max_dec = math.ceil(B_total / world) if B_total else 0

    # N > 1: the step's results (decode outputs, prefill final states) land on
    # rank 0.  With --gather peer every rank's kernels store them straight
    # into rank 0's rank-major buffers (CUDA IPC mapping, plain stores over
    # NVLink while the step computes) and one 4-byte all-reduce closes the
    # step; with --gather nccl (or if any rank cannot map) an NCCL gather
    # runs after the compute.
    dec_peer = fin_peer = None
    gather_mode = "none" if world == 1 else args.gather
    if world > 1 and args.gather == "peer":
        try:
            if B_total:
                dec_peer = shard.PeerResult(
                    [len(range(B_total)[shard.block_partition(B_total, world, r)])
                     for r in range(world)], (Tdec, HV, D), torch.bfloat16, dev)
            if wl["prefill"]:
                fin_peer = shard.PeerResult(seq_counts, (HV, D, D), torch.float32, dev)
        except RuntimeError as e:
            if dec_peer is not None:
                dec_peer.close()
            dec_peer = fin_peer = None
            gather_mode = f"nccl (peer mapping failed: {e})"
    peer = dec_peer or fin_peer
    total_tokens = B_total * Tdec + total_prefill_tokens
    stream = torch.cuda.current_stream(dev)

    ev = {k: [] for k in ("s", "d", "p", "g")}
    # per-kernel events inside each timed prefill call (recorded by the
    # library right after each of its launches, on this stream)
    n_pre_launch = (gdn._native.prefill_kernel_launches(pre["T"], pre["N"])
                    if pre is not None and pre["N"] > 0 else 0)
    ev["k"] = []

    # decode and prefill are independent: with overlap on, decode runs on a
    # side stream next to the prefill (its CTAs fill SMs the prefill leaves
    # idle) and the step joins both before the gather
    overlap = args.overlap == "on" and dec is not None and pre is not None and pre["N"] > 0
    side = torch.cuda.Stream(dev) if overlap else stream
    ev["dside"] = []

    def decode(dec_dst):
        with torch.cuda.stream(side):
            run_decode(gdn, dec, A_log, dt_bias, dec_dst)

    def step(record):
        # this step's destinations (the peer results alternate two buffers)
        dec_dst = dec_peer.rows_for_me() if dec_peer is not None else dec_out
        fin_dst = fin_peer.rows_for_me() if fin_peer is not None else (pre["final"] if pre else None)
        if record:
            e = torch.cuda.Event(enable_timing=True)
            e.record(stream)
            ev["s"].append(e)
        if overlap:
            side.wait_stream(stream)
        if dec is not None and not overlap:
            decode(dec_dst)
        if record:
            e = torch.cuda.Event(enable_timing=True)
            e.record(stream)
            ev["d"].append(e)
        if pre is not None and pre["N"] > 0:
            kev = None
            if record and not overlap:
                kev = [torch.cuda.Event(enable_timing=True) for _ in range(n_pre_launch)]
                ev["k"].append(kev)
            gdn.prefill.prefill_into(pre["q"], pre["k"], pre["v"], pre["h0"], A_log, pre["a"],
                                     dt_bias, pre["b"], pre["cu"], None, pre["out"],
                                     fin_dst, pre["ws"], events=kev)
        if overlap:
            # issued after the prefill, so its CTAs take the SMs the prefill's
            # kernels leave free (their tails and the gaps between them)
            decode(dec_dst)
            if record:
                e = torch.cuda.Event(enable_timing=True)
                e.record(side)
                ev["dside"].append(e)
            stream.wait_stream(side)
        if record:
            e = torch.cuda.Event(enable_timing=True)
            e.record(stream)
            ev["p"].append(e)
        if peer is not None:
            # one all-reduce closes the step for both results (same group, stream)
            peer.publish(*[r for r in (dec_peer, fin_peer) if r is not None and r is not peer])
        elif world > 1:
            if dec_out is not None or max_dec:
                t = dec_out if dec_out is not None else torch.empty(0, Tdec, HV, D, dtype=torch.bfloat16, device=dev)
                shard.gather_padded(t, max_dec)
            if max_seqs:
                t = pre["final"] if pre is not None else torch.empty(0, HV, D, D, device=dev)
                shard.gather_padded(t, max_seqs)
        if record:
            e = torch.cuda.Event(enable_timing=True)
            e.record(stream)
            ev["g"].append(e)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize(dev)

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        step(False)
    barrier()
    sampler = ClockSampler(True, local_rank)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    barrier()
    t0.record(stream)
    for _ in range(args.steps):
        step(True)
    t1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    clocks = merge_clocks(dist, world, sampler.stop())
    elapsed_ms = max_over_ranks(t0.elapsed_time(t1))
    ms_step = elapsed_ms / args.steps
    # with overlap the decode runs beside the prefill: its phase is from the
    # step start to its own end, and the prefill's from the step start
    d_ms = np.mean([a.elapsed_time(b) for a, b in zip(ev["s"], ev["dside" if overlap else "d"])])
    p_ms = np.mean([a.elapsed_time(b) for a, b in zip(ev["s" if overlap else "d"], ev["p"])])
    g_ms = np.mean([a.elapsed_time(b) for a, b in zip(ev["p"], ev["g"])])
    d_ms_max, p_ms_max, g_ms_max = (max_over_ranks(float(x)) for x in (d_ms, p_ms, g_ms))
    status = gdn._native.read_device_status()
    if status:
        raise SystemExit(f"device status {status} after the timed region")

    # per-kernel mean durations of the prefill call (CUDA events the library
    # records after each of its launches), max over ranks
    # (one fixed-size reduction on every rank, whatever its own launch count)
    knames = ["meta", "prep", "scan", "compose", "scan_pass3"]
    local = np.full(len(knames), -1.0)
    for i in range(min(n_pre_launch, len(knames)) if ev["k"] else 0):
        durs = [(st if i == 0 else ks[i - 1]).elapsed_time(ks[i]) for st, ks in zip(ev["d"], ev["k"])]
        local[i] = float(np.mean(durs))
    if world > 1:
        t = torch.tensor(local, dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        local = t.cpu().numpy()
    kernel_ms = {n: float(x) for n, x in zip(knames, local) if x >= 0}

    peaks = load_peaks()
    execution = {
        "streams": ("decode on a side stream next to the prefill, joined each step" if overlap
                    else "one stream (decode, then prefill)"),
        "results": ("kernels store decode outputs + prefill final states into rank 0's buffers "
                    "over NVLink (CUDA IPC), one 4-byte all-reduce per step" if peer is not None else
                    "NCCL gather of decode outputs + prefill final states to rank 0"
                    if world > 1 else "single GPU, results stay in place"),
        "gather": gather_mode,
    }
    result = {
        "metric": "GDN serving throughput (decode + prefill tokens/s, max-over-ranks device time)",
        "value": total_tokens / (ms_step / 1e3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_step,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded; the benchmark configs' value distributions)",
        "config": workload_config(args.workload, world),
        "execution": execution,
        "gpu_launches": args.steps * ((1 if dec is not None else 0) + n_pre_launch),
        "phases_ms": {"decode": d_ms_max, "prefill": p_ms_max, "gather": g_ms_max},
        "prefill_kernels_ms": kernel_ms,
        "clocks": clocks,
    }
    if dec is not None:
        state_bytes = DECODE_STATE_BYTES // 2 if wl.get("state_bf16") else DECODE_STATE_BYTES
        gbs = B * (state_bytes + Tdec * DECODE_VEC_BYTES) / (d_ms / 1e3) / 1e9
        result["decode"] = {"us_per_step": d_ms_max * 1e3, "state_gbs_rank0": gbs,
                            "batch_per_rank": B}
        result["roofline_decode"] = {
            "bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": gbs / peaks["hbm_gbs"],
            "traffic": load_traffic(args.workload).get("decode_bytes_per_launch"),
            "peak_source": peaks["source"] + " hbm copy"}
    if pre is not None:
        flops = pre["T"] * PREFILL_FLOP_PER_TOKEN
        tflops = flops / (p_ms / 1e3) / 1e12
        n_states = pre["N"] * (2 if pre["h0"] is not None else 1)   # h0 read (if given), final written
        result["prefill"] = {"tokens_per_s": total_prefill_tokens / (p_ms_max / 1e3),
                             "tflops_rank0": tflops, "tokens_rank0": pre["T"]}
        traffic = load_traffic(args.workload)
        # the prefill call (all its launches) is the hot path's one "launch";
        # the timed region is well under a second, so the burst peaks apply
        result["roofline"] = roofline_entry(
            "prefill call (meta + prep + scan" + (" + compose + scan pass 3" if n_pre_launch == 5 else "")
            + " launches)", flops, pre["T"] * PREFILL_BYTES_PER_TOKEN + n_states * STATE_BYTES,
            p_ms / 1e3, peaks, traffic.get("prefill_bytes_per_launch"))
        per_kernel = {}
        if "prep" in kernel_ms:
            per_kernel["prep"] = roofline_entry(
                "gdn_prefill_prep_kernel", pre["T"] * PREP_FLOP_PER_TOKEN,
                pre["T"] * PREP_BYTES_PER_TOKEN, kernel_ms["prep"] / 1e3, peaks,
                traffic.get("prep_bytes_per_launch"))
        if "scan" in kernel_ms:
            scan_s = (kernel_ms["scan"] + kernel_ms.get("scan_pass3", 0.0)) / 1e3
            per_kernel["scan"] = roofline_entry(
                "gdn_prefill_scan_kernel" + (" (both passes)" if "scan_pass3" in kernel_ms else ""),
                pre["T"] * SCAN_FLOP_PER_TOKEN,
                pre["T"] * SCAN_BYTES_PER_TOKEN + n_states * STATE_BYTES, scan_s, peaks,
                traffic.get("scan_bytes_per_launch"))
        # tensor-pipe utilisation (sm__pipe_tensor_cycles_active, % of active
        # cycles) of each kernel from its one-kernel ncu capture; the call's
        # figure is their average weighted by this run's kernel times
        tc = {k: traffic.get(f"{k}_tensor_pipe_active_pct") for k in per_kernel}
        for k, v in tc.items():
            per_kernel[k]["tensor_pipe_active_pct"] = v
        if per_kernel and all(v is not None for v in tc.values()):
            w = {k: per_kernel[k]["measured_ms"] for k in per_kernel}
            result["roofline"]["tensor_pipe_active_pct"] = (
                sum(tc[k] * w[k] for k in w) / sum(w.values()))
            result["roofline"]["tensor_pipe_source"] = (
                "ncu one-kernel captures (profiles/traffic.json), weighted by this run's kernel times")
        if per_kernel:
            result["roofline_kernels"] = per_kernel
    elif dec is not None:
        result["roofline"] = result.pop("roofline_decode")

    # ---- end to end through the public entry points with host buffers ----
    if not args.no_e2e:
        result["e2e"] = e2e_run(torch, gdn, args, dec, pre, A_log, dt_bias, dev, world,
                                max_over_ranks, barrier, total_tokens)

    if world == 1 and not args.no_triton:
        ours = {"step_ms": ms_step, "decode_ms": d_ms_max, "prefill_ms": p_ms_max}
        try:
            result["triton_reference"] = triton_reference_block(
                torch, gdn, args, dev, A_log, dt_bias, dec, pre, ours)
        except Exception as e:  # noqa: BLE001 -- the reference's kernels are not ours to fix
            result["triton_reference"] = {"unavailable": f"{type(e).__name__}: {e}"[:300]}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(args.workload, budget_s=args.cpu_seconds)
    for res in (dec_peer, fin_peer):
        if res is not None:
            res.close()
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()
    if rank == 0:
        emit(result)


def bwd_arm(args):
    """Training step of the prefill: one backward call (recompute + reverse
    scan + chunk gradients) per step over the workload's sequences, inputs
    and d_out resident.  N > 1: sequences sharded by LPT, and the only
    exchange a training step has here, the sum of the [8] parameter
    gradients dA_log and ddt_bias over ranks (NCCL all-reduce)."""
    import torch
    import torch.distributed as dist
    from importlib import import_module

    gdn = importlib.import_module("track-c-gdn_b200")
    shard = import_module("track-c-gdn_b200.shard")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        os.environ.setdefault("NCCL_DEBUG", "WARN")
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)
    wl = WORKLOADS[args.workload]
    lengths = prefill_lengths(wl["prefill"])
    parts = shard.lpt_partition(lengths.tolist(), world)
    my = lengths[parts[rank]]
    with_state = wl["prefill"] == "c3"
    pre = make_prefill_inputs(torch, my, with_state, 300 + rank, dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(7)
    A_log = (torch.rand(HV, generator=gen, device=dev) * 2.7).float()
    dt_bias = (torch.randn(HV, generator=gen, device=dev) * 0.1).float()
    T, N = pre["T"], pre["N"]
    d_out = (torch.randn(T, HV, D, generator=gen, device=dev) * 0.1).bfloat16()
    d_final = (torch.randn(N, HV, D, D, generator=gen, device=dev) * 0.01) if with_state else None
    f32 = dict(dtype=torch.float32, device=dev)
    outs = [torch.empty(T, HQK, D, **f32), torch.empty(T, HQK, D, **f32),
            torch.empty(T, HV, D, **f32), torch.empty(T, HV, **f32), torch.empty(T, HV, **f32),
            torch.empty(HV, **f32), torch.empty(HV, **f32),
            torch.empty(N, HV, D, D, **f32) if with_state else None]
    ws = gdn.prefill.alloc_backward_workspace(T, N, dev)
    stream = torch.cuda.current_stream(dev)
    params = torch.empty(2 * HV, **f32)

    def step():
        gdn.prefill.backward_into(pre["q"], pre["k"], pre["v"], pre["h0"], A_log, pre["a"],
                                  dt_bias, pre["b"], pre["cu"], None, d_out, d_final, *outs, ws)
        if world > 1:
            params[:HV].copy_(outs[5])
            params[HV:].copy_(outs[6])
            dist.all_reduce(params)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize(dev)

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        step()
    barrier()
    sampler = ClockSampler(True, local_rank)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    barrier()
    t0.record(stream)
    for _ in range(args.steps):
        step()
    t1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    clocks = merge_clocks(dist, world, sampler.stop())
    ms = max_over_ranks(t0.elapsed_time(t1)) / args.steps
    status = gdn._native.read_device_status()
    if status:
        raise SystemExit(f"device status {status} after the timed region")
    total = int(lengths.sum())
    tflops = T * BWD_FLOP_PER_TOKEN / (ms / 1e3) / 1e12
    peaks = load_peaks()
    result = {
        "metric": "GDN prefill backward throughput (tokens/s, max-over-ranks device time)",
        "value": total / (ms / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "fp32 (backward kernels; recompute bf16 MMAs)",
        "data": "synthetic (seeded; the benchmark configs' value distributions)",
        "config": {"workload": wl["desc"], "prefill_sequences": len(lengths),
                   "prefill_tokens": total,
                   "l2": "inputs larger than L2 (no flush needed)",
                   "parallelism": f"shard{world}: LPT by sequence" +
                                  ("; NCCL all-reduce of dA_log, ddt_bias" if world > 1 else "")},
        "gpu_launches": args.steps * gdn._native.lib.gdn_prefill_backward_kernel_launches(),
        "roofline": {"kernel": "whole backward call (recompute + reverse scan + chunk gradients)",
                     "bound": "tensor", "achieved": tflops,
                     "peak": peaks["bf16_tflops_sustained"], "unit": "TFLOP/s",
                     "frac": tflops / peaks["bf16_tflops_sustained"], "traffic": None,
                     "flop_per_token": BWD_FLOP_PER_TOKEN,
                     "peak_source": peaks["source"] + " bf16 sustained"},
        "clocks": clocks,
    }
    if not args.no_e2e:
        # end to end: inputs from pinned host memory, gradients back, serial
        keys = [x for x in ("q", "k", "v", "a", "b", "cu", "h0") if pre.get(x) is not None]
        host = {x: pre[x].cpu().pin_memory() for x in keys}
        host["d_out"] = d_out.cpu().pin_memory()
        if d_final is not None:
            host["d_final"] = d_final.cpu().pin_memory()
        devb = {x: torch.empty_like(t, device=dev) for x, t in host.items()}
        host_out = [None if o is None else torch.empty(o.shape, dtype=o.dtype).pin_memory()
                    for o in outs]
        h2d = sum(t.numel() * t.element_size() for t in host.values())
        d2h = sum(o.numel() * o.element_size() for o in outs if o is not None)

        def e2e_step():
            for x, t in host.items():
                devb[x].copy_(t, non_blocking=True)
            gdn.prefill.backward_into(devb["q"], devb["k"], devb["v"], devb.get("h0"), A_log,
                                      devb["a"], dt_bias, devb["b"], devb["cu"], None,
                                      devb["d_out"], devb.get("d_final"), *outs, ws)
            for o, h in zip(outs, host_out):
                if o is not None:
                    h.copy_(o, non_blocking=True)

        e2e_step()
        barrier()
        n = max(2, min(args.steps, args.e2e_steps))
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        ems = max_over_ranks(e0.elapsed_time(e1)) / n
        result["e2e"] = {"value": total / (ems / 1e3), "unit": "tokens/s", "ms_per_step": ems,
                         "steps": n, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                         "api": "prefill.backward_into, pinned host buffers, one stream",
                         "bytes_per_step_note": "per rank" if world > 1 else "single GPU"}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = bwd_cpu_baseline(lengths, budget_s=args.cpu_seconds)
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()
    if rank == 0:
        emit(result)


def bwd_cpu_baseline(lengths, budget_s: float = 15.0):
    """Autograd of the restated token recurrence (oracle/autograd_ref.py) in
    fp32 on the host cores, over whole sequences drawn from the workload
    until the budget is spent; extrapolated per token."""
    import torch
    from oracle import autograd_ref
    rng = np.random.default_rng(0)
    toks, secs, n = 0, 0.0, 0
    t_start = time.perf_counter()
    while time.perf_counter() - t_start < budget_s and n < len(lengths):
        L = int(min(lengths[n], 512))
        n += 1
        x = {k: torch.from_numpy(rng.standard_normal(s).astype(np.float32))
             for k, s in (("q", (L, HQK, D)), ("k", (L, HQK, D)), ("v", (L, HV, D)),
                          ("a", (L, HV)), ("b", (L, HV)))}
        A_log = torch.rand(HV)
        dt = torch.randn(HV) * 0.1
        d_out = torch.randn(L, HV, D) * 0.1
        t0 = time.perf_counter()
        autograd_ref.prefill_grads(x["q"], x["k"], x["v"], None, A_log, x["a"], dt, x["b"],
                                   [0, L], None, d_out, None, dtype=torch.float32)
        secs += time.perf_counter() - t0
        toks += L
    return {"value": toks / secs, "unit": "tokens/s", "cores": torch.get_num_threads(),
            "kind": "port", "sample": f"{n} sequences (first {toks} tokens, at most 512 per "
            "sequence) of the workload: torch autograd of the restated recurrence, fp32",
            "wall_s": round(time.perf_counter() - t_start, 1)}


def e2e_run(torch, gdn, args, dec, pre, A_log, dt_bias, dev, world, max_over_ranks, barrier,
            total_tokens):
    """The step as a serving loop would run it through the public entry points,
    from pinned host memory and back.  Every step copies its inputs host ->
    device and its outputs (decode out, prefill out, final states) device ->
    host inside the timed region.  Double buffered: step s+1's inputs cross
    PCIe on a copy-in stream while step s computes, and step s's outputs cross
    back on a copy-out stream (PCIe is full duplex); events keep each buffer
    slot from being overwritten before its last reader is done.  Compute uses
    decode.decode_into (state updated in place) and prefill.prefill_into (no
    host synchronisation).  The same step run serially on one stream is
    reported beside it."""
    steps = max(2, min(args.steps, args.e2e_steps))
    comp = torch.cuda.current_stream(dev)
    s_in = torch.cuda.Stream(dev)
    s_out = torch.cuda.Stream(dev)
    dec_keys = ("q", "k", "v", "a", "b")
    pre_keys = ("q", "k", "v", "a", "b", "cu") + (("h0",) if pre is not None and pre["h0"] is not None else ())
    host_in, dev_in, host_out, dev_out = {}, [{}, {}], [{}, {}], [{}, {}]
    h2d = d2h = 0
    if dec is not None:
        for key in dec_keys:
            host_in["d" + key] = dec[key].cpu().pin_memory()
            h2d += dec[key].numel() * dec[key].element_size()
        for sl in range(2):
            for key in dec_keys:
                dev_in[sl]["d" + key] = torch.empty_like(dec[key])
            dev_out[sl]["dout"] = torch.empty(dec["B"], dec["T"], HV, D, dtype=torch.bfloat16,
                                              device=dev)
            host_out[sl]["dout"] = torch.empty(dec["B"], dec["T"], HV, D,
                                               dtype=torch.bfloat16).pin_memory()
        d2h += dec["B"] * dec["T"] * HV * D * 2
    if pre is not None and pre["N"] > 0:
        for key in pre_keys:
            host_in["p" + key] = pre[key].cpu().pin_memory()
            h2d += pre[key].numel() * pre[key].element_size()
        for sl in range(2):
            for key in pre_keys:
                dev_in[sl]["p" + key] = torch.empty_like(pre[key])
            dev_out[sl]["pout"] = torch.empty(pre["T"], HV, D, dtype=torch.bfloat16, device=dev)
            dev_out[sl]["pfin"] = torch.empty(pre["N"], HV, D, D, dtype=torch.float32, device=dev)
            host_out[sl]["pout"] = torch.empty(pre["T"], HV, D, dtype=torch.bfloat16).pin_memory()
            host_out[sl]["pfin"] = torch.empty(pre["N"], HV, D, D, dtype=torch.float32).pin_memory()
        d2h += pre["T"] * HV * D * 2 + pre["N"] * HV * D * D * 4
    ev = {name: [torch.cuda.Event(), torch.cuda.Event()] for name in ("in", "comp", "out")}

    def compute(sl):
        t = dev_in[sl]
        if dec is not None:
            d = dict(dec, q=t["dq"], k=t["dk"], v=t["dv"], a=t["da"], b=t["db"])
            run_decode(gdn, d, A_log, dt_bias, dev_out[sl]["dout"])
        if pre is not None and pre["N"] > 0:
            gdn.prefill.prefill_into(t["pq"], t["pk"], t["pv"], t.get("ph0"), A_log, t["pa"],
                                     dt_bias, t["pb"], t["pcu"], None, dev_out[sl]["pout"],
                                     dev_out[sl]["pfin"], pre["ws"])

    def pipelined(n):
        for s in range(n):
            sl = s % 2
            with torch.cuda.stream(s_in):
                if s >= 2:
                    s_in.wait_event(ev["comp"][sl])  # step s-2 no longer reads this input slot
                for key, h in host_in.items():
                    dev_in[sl][key].copy_(h, non_blocking=True)
                ev["in"][sl].record(s_in)
            comp.wait_event(ev["in"][sl])
            if s >= 2:
                comp.wait_event(ev["out"][sl])  # step s-2's outputs have left this slot
            compute(sl)
            ev["comp"][sl].record(comp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev["comp"][sl])
                for key, d in dev_out[sl].items():
                    host_out[sl][key].copy_(d, non_blocking=True)
                ev["out"][sl].record(s_out)

    def serial(n):
        for s in range(n):
            for key, h in host_in.items():
                dev_in[0][key].copy_(h, non_blocking=True)
            compute(0)
            for key, d in dev_out[0].items():
                host_out[0][key].copy_(d, non_blocking=True)

    def timed(fn, n):
        torch.cuda.synchronize(dev)
        barrier()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(comp)
        s_in.wait_stream(comp)
        fn(n)
        s_out.wait_stream(comp)
        comp.wait_stream(s_out)
        t1.record(comp)
        torch.cuda.synchronize(dev)
        barrier()
        return max_over_ranks(t0.elapsed_time(t1)) / n

    pipelined(2)  # warm-up
    ms = timed(pipelined, steps)
    ms_serial = timed(serial, steps)
    return {"value": total_tokens / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms,
            "steps": steps, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "api": "decode.decode_into (state in place) + prefill.prefill_into, pinned host "
                   "buffers, double-buffered copy-in / copy-out streams",
            "serial_ms_per_step": ms_serial,
            "serial_value": total_tokens / (ms_serial / 1e3),
            "bytes_per_step_note": "per rank" if world > 1 else "single GPU"}


# ---------------------------------------------------------------------------
# CPU oracle (reported baseline and the reference arm)
# ---------------------------------------------------------------------------
def _bf16_bits(x: np.ndarray) -> np.ndarray:
    # round to nearest even; 32-bit arithmetic cannot overflow for finite inputs
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    return ((u + np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1))) >> 16).astype(np.uint16)


def _cpu_decode_inputs(rng, B, T=1):
    def nrm(s):
        x = rng.standard_normal(s, dtype=np.float32)
        return x / np.linalg.norm(x, axis=-1, keepdims=True)
    return dict(q=_bf16_bits(nrm((B, T, HQK, D))), k=_bf16_bits(nrm((B, T, HQK, D))),
                v=_bf16_bits(rng.standard_normal((B, T, HV, D), dtype=np.float32)),
                a=_bf16_bits(rng.standard_normal((B, T, HV), dtype=np.float32)),
                b=_bf16_bits(rng.standard_normal((B, T, HV), dtype=np.float32)),
                state=(rng.standard_normal((B, HV, D, D), dtype=np.float32) * 0.02))


def _cpu_prefill_inputs(rng, lengths, with_state):
    T = int(np.sum(lengths))
    cu = np.zeros(len(lengths) + 1, np.int64)
    cu[1:] = np.cumsum(lengths)

    def nrm(s):
        x = rng.standard_normal(s, dtype=np.float32)
        return x / np.linalg.norm(x, axis=-1, keepdims=True)
    return dict(q=_bf16_bits(nrm((T, HQK, D))), k=_bf16_bits(nrm((T, HQK, D))),
                v=_bf16_bits(rng.standard_normal((T, HV, D), dtype=np.float32)),
                a=_bf16_bits(rng.standard_normal((T, HV), dtype=np.float32)),
                b=_bf16_bits(rng.standard_normal((T, HV), dtype=np.float32)),
                state=(rng.standard_normal((len(lengths), HV, D, D), dtype=np.float32) * 0.02)
                if with_state else None, cu=cu, T=T)


class CpuStepSampler:
    """Times the CPU oracle (the reference recurrence restated in C, OpenMP
    over all host threads) on sample steps of a workload.  Sample step j is
    1/k of the workload's step with the same decode : prefill mix: decode of
    B/k requests (T tokens each) and prefill of the sequences j mod k,
    j mod k + k, j mod k + 2k, ... of the workload's length list.  Its tokens/s
    is therefore that of the full step's mix, measured directly (nothing is
    extrapolated); the full step would take about k times one sample step."""

    def __init__(self, workload: str):
        import oracle
        self.oracle = oracle
        self.threads = oracle.default_threads()
        self.wl = WORKLOADS[workload]
        self.lengths = prefill_lengths(self.wl["prefill"]) if self.wl["prefill"] else None
        B = self.wl["decode_batch"]
        if self.lengths is not None:
            self.k = 64 if len(self.lengths) >= 64 else 1
        else:
            self.k = max(1, B // 64)
        self.dec_req = B // self.k if B else 0
        self.dec_T = self.wl.get("decode_tokens", 1)
        self.rng = np.random.default_rng(77)
        self.A_log = (self.rng.random(HV, dtype=np.float32) * 2.7).astype(np.float32)
        self.dt = (self.rng.standard_normal(HV, dtype=np.float32) * 0.1).astype(np.float32)
        self.j = 0
        self.times = []      # seconds per timed sample step
        self.tokens = []     # tokens per timed sample step
        self.seqs_seen = set()

    def step(self, record: bool = True):
        tok, secs = 0, 0.0
        if self.dec_req:
            inp = _cpu_decode_inputs(self.rng, self.dec_req, self.dec_T)
            fn = self.oracle.decode if self.dec_T == 1 else self.oracle.decode_mtp
            t = time.perf_counter()
            fn(inp["q"], inp["k"], inp["v"], inp["state"], self.A_log, inp["a"], self.dt, inp["b"],
               nthreads=self.threads)
            secs += time.perf_counter() - t
            tok += self.dec_req * self.dec_T
        if self.lengths is not None:
            idx = list(range(self.j % self.k, len(self.lengths), self.k))
            inp = _cpu_prefill_inputs(self.rng, self.lengths[idx], self.wl["prefill"] == "c3")
            t = time.perf_counter()
            self.oracle.prefill(inp["q"], inp["k"], inp["v"], inp["state"], self.A_log, inp["a"],
                                self.dt, inp["b"], inp["cu"], nthreads=self.threads)
            secs += time.perf_counter() - t
            tok += inp["T"]
            if record:
                self.seqs_seen.update(idx)
        self.j += 1
        if record:
            self.times.append(secs)
            self.tokens.append(tok)

    def value(self) -> float:
        return float(sum(self.tokens) / sum(self.times))

    def ms_per_step(self) -> float:
        return float(np.mean(self.times) * 1e3)

    def describe(self) -> str:
        parts = []
        if self.dec_req:
            parts.append(f"decode of {self.dec_req} requests x {self.dec_T} token(s)")
        if self.lengths is not None:
            per = len(range(0, len(self.lengths), self.k))
            parts.append(f"prefill of {per} sequence(s) (every {self.k}th of the workload's "
                         f"{len(self.lengths)}-sequence length list)")
        frac = f"1/{self.k} of the workload's step" if self.k > 1 else "the whole workload step"
        seen = (f"; the timed steps covered {len(self.seqs_seen)} of the {len(self.lengths)} "
                "sequences" if self.lengths is not None else "")
        return (f"each step = {frac} with the same decode:prefill mix: " + " + ".join(parts)
                + f"; {len(self.times)} timed steps, {sum(self.tokens)} tokens" + seen)


def cpu_baseline(workload: str, budget_s: float = 15.0):
    """The oracle on sample steps for about `budget_s` seconds (at least two)."""
    sampler = CpuStepSampler(workload)
    t_start = time.perf_counter()
    sampler.step(record=False)  # warm-up (page-in, thread pool)
    while len(sampler.times) < 2 or time.perf_counter() - t_start < budget_s:
        sampler.step()
    return {"value": sampler.value(), "unit": "tokens/s", "cores": sampler.threads,
            "kind": "port", "sample": sampler.describe(),
            "ms_per_sample_step": sampler.ms_per_step(),
            "wall_s": round(time.perf_counter() - t_start, 1)}


def reference_arm(args):
    """The reference's path on the host cores: the CPU restatement of its
    recurrence (the reference's own code is Python/Triton and GPU-only).
    Rank 0 alone runs; W warm-up and K timed sample steps (see
    CpuStepSampler), so `steps` and `ms_per_step` describe exactly what was
    timed."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    sampler = CpuStepSampler(args.workload)
    for _ in range(args.warmup):
        sampler.step(record=False)
    t_start = time.perf_counter()
    for _ in range(args.steps):
        sampler.step()
    value = sampler.value()
    cpu = {"value": value, "unit": "tokens/s", "cores": sampler.threads, "kind": "port",
           "sample": sampler.describe(), "wall_s": round(time.perf_counter() - t_start, 1)}
    emit({
        "impl": "reference",
        "metric": "GDN serving throughput (decode + prefill tokens/s, max-over-ranks device time)",
        "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": sampler.ms_per_step(), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (seeded; the benchmark configs' value distributions)",
        "config": workload_config(args.workload, world),
        "execution": {"where": f"rank 0's host cores ({sampler.threads} threads)",
                      "step": f"1/{sampler.k} of the workload step per timed step",
                      "full_step_ms_estimate": sampler.ms_per_step() * sampler.k},
        "cpu_baseline": cpu,
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "the reference's path is Python/Triton (GPU only); its CPU implementation "
                "is the oracle's C restatement of the same recurrence (OpenMP, all host threads)",
    })


TRITON_REF_DIR = ROOT / "baseline" / "_ref"


def _load_triton_ref(definition: str):
    """Import the reference's Triton solution `<definition>/solution/triton/
    kernel.py` from the unmodified copy staged under baseline/_ref (the
    reference is not pip-installable)."""
    import importlib.util
    path = TRITON_REF_DIR / definition / "solution" / "triton" / "kernel.py"
    if not path.exists():
        return None
    spec = importlib.util.spec_from_file_location(f"triton_ref_{definition}", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _flush_l2(torch, buf):
    buf.add_(1)  # writes 256 MiB (more than the 126 MB L2)


def _time_calls(torch, stream, fn, n, flush=None):
    """Mean device time (ms) of `fn` over n calls, CUDA events on `stream`
    around each call only (an L2 flush, when given, runs before each call
    outside the events)."""
    pairs = []
    for _ in range(n):
        if flush is not None:
            flush()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        fn()
        e1.record(stream)
        pairs.append((e0, e1))
    torch.cuda.synchronize()
    return float(np.mean([a.elapsed_time(b) for a, b in pairs]))


def triton_reference_block(torch, gdn, args, dev, A_log, dt_bias, dec, pre, ours):
    """The reference's own Triton kernels (its two solution/triton/kernel.py
    files, unmodified, staged under baseline/_ref) timed on this GPU on the
    same inputs as this run (N = 1): the workload's step and its phases, and
    for the default workload also C2 (one 4,096-token sequence, the north
    star's T >= 4096 case), against ours on the same inputs.  Speed-up =
    reference ms / ours."""
    dec_mod = _load_triton_ref("gdn_decode_qk4_v8_d128_k_last") if dec is not None else None
    pre_mod = _load_triton_ref("gdn_prefill_qk4_v8_d128_k_last")
    if (dec is not None and dec_mod is None) or pre_mod is None:
        return {"unavailable": f"reference Triton solutions not staged under {TRITON_REF_DIR}"}
    if dec is not None and (dec["T"] != 1 or dec.get("bf16")):
        return {"unavailable": "the reference decode takes one fp32-state token per request; "
                               "bench.py --impl triton times it token by token"}
    stream = torch.cuda.current_stream(dev)
    n = max(3, min(args.steps, 10))
    out = {"source": "solution/triton/kernel.py (prefill) and gdn_decode_qk4_v8_d128_k_last/"
                     "solution/triton/kernel.py (decode), unmodified, through their run() entry "
                     "points; CUDA events, same inputs and GPU as this run",
           "steps": n}

    def ref_decode():
        return dec_mod.run(dec["q"], dec["k"], dec["v"], dec["state"], A_log, dec["a"], dt_bias,
                           dec["b"], None)

    def ref_prefill(p):
        return pre_mod.run(p["q"], p["k"], p["v"], p["h0"], A_log, p["a"], dt_bias, p["b"],
                           p["cu"], None)

    def entry(ref_ms, our_ms):
        return {"reference_triton": ref_ms, "b200": our_ms, "speedup": ref_ms / our_ms}

    for _ in range(3):  # warm-up, JIT compilation included
        if dec is not None:
            ref_decode()
        if pre is not None and pre["N"] > 0:
            ref_prefill(pre)
    torch.cuda.synchronize()
    phases = {}
    if dec is not None:
        phases["decode"] = _time_calls(torch, stream, ref_decode, n)
        out[f"decode_b{dec['B']}_ms"] = entry(phases["decode"], ours["decode_ms"])
    if pre is not None and pre["N"] > 0:
        phases["prefill"] = _time_calls(torch, stream, lambda: ref_prefill(pre), n)
        out["prefill_ms"] = entry(phases["prefill"], ours["prefill_ms"])
        # parity of the two on these inputs (final states; outputs by median
        # per-token distance, the reference's output stage being nondeterministic)
        o_ref, s_ref = ref_prefill(pre)
        o, s = gdn.prefill.run(pre["q"], pre["k"], pre["v"], pre["h0"], A_log, pre["a"], dt_bias,
                               pre["b"], pre["cu"], None)
        tok = ((o.float() - o_ref.float()).flatten(1).norm(dim=1)
               / o_ref.float().flatten(1).norm(dim=1).clamp_min(1e-30))
        out["prefill_parity"] = {
            "final_state_rel_fro": float((s - s_ref).norm() / s_ref.norm().clamp_min(1e-30)),
            "out_token_rel_median": float(tok.median())}
        del o_ref, s_ref, o, s
    out["step_ms"] = entry(sum(phases.values()), ours["step_ms"])
    if args.workload == "c4":
        # C2: T = 4096 in one sequence, zero initial state (L2 flushed before each call)
        c2 = make_prefill_inputs(torch, prefill_lengths("c2"), False, 200, dev)
        o2 = torch.empty(c2["T"], HV, D, dtype=torch.bfloat16, device=dev)
        f2 = torch.empty(c2["N"], HV, D, D, dtype=torch.float32, device=dev)
        ws2 = gdn.prefill.alloc_workspace(c2["T"], c2["N"], dev)
        flush_buf = torch.empty(64 << 20, dtype=torch.float32, device=dev)

        def ours_c2():
            gdn.prefill.prefill_into(c2["q"], c2["k"], c2["v"], None, A_log, c2["a"], dt_bias,
                                     c2["b"], c2["cu"], None, o2, f2, ws2)

        for _ in range(3):
            ours_c2()
            ref_prefill(c2)
        flush = lambda: _flush_l2(torch, flush_buf)  # noqa: E731
        m = max(n, 20)
        out["c2_prefill_ms"] = entry(_time_calls(torch, stream, lambda: ref_prefill(c2), m, flush),
                                     _time_calls(torch, stream, ours_c2, m, flush))
        out["c2_prefill_ms"]["l2"] = "flushed before each call"
    pre_keys = [k for k in ("prefill_ms", "c2_prefill_ms") if k in out]
    out["prefill_faster_than_reference_at_T_ge_4096"] = (
        all(out[k]["speedup"] > 1.0 for k in pre_keys) if pre_keys else None)
    return out


def triton_arm(args):
    """The reference's own Triton kernels on this GPU, through their `run`
    entry points, on the same seeded inputs as the b200 arm at N=1 (decode:
    value-returning run, which allocates new_state as the reference does;
    prefill: run, including its host-side checks).  Also reports how far our
    outputs are from the Triton outputs on these inputs."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    wl = WORKLOADS[args.workload]
    dec_mod = _load_triton_ref("gdn_decode_qk4_v8_d128_k_last") if wl["decode_batch"] else None
    pre_mod = _load_triton_ref("gdn_prefill_qk4_v8_d128_k_last") if wl["prefill"] else None
    if (wl["decode_batch"] and dec_mod is None) or (wl["prefill"] and pre_mod is None):
        emit({"impl": "triton-reference",
              "unavailable": f"reference Triton solutions not staged under {TRITON_REF_DIR}"})
        return
    import torch
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev)
    g.manual_seed(1234)  # the b200 arm's rank-0 seeds, so both arms see the same inputs
    A_log = (torch.rand(HV, generator=g, device=dev) * 2.7).float()
    dt_bias = (torch.randn(HV, generator=g, device=dev) * 0.1).float()
    Tdec = wl.get("decode_tokens", 1)
    dec = (make_decode_inputs(torch, wl["decode_batch"], 100, dev, Tdec, wl.get("state_bf16", False))
           if wl["decode_batch"] else None)
    pre = None
    if wl["prefill"]:
        lengths = prefill_lengths(wl["prefill"])
        pre = make_prefill_inputs(torch, lengths, wl["prefill"] == "c3", 200, dev)
    stream = torch.cuda.current_stream(dev)
    ev = {k: [] for k in ("s", "d", "p")}
    keep = {}
    # the reference keeps fp32 state: a bf16 state is widened once, outside the timing
    ref_state = dec["state"].float() if dec is not None else None

    def step(record):
        if record:
            ev["s"].append(torch.cuda.Event(enable_timing=True))
            ev["s"][-1].record(stream)
        if dec is not None:
            # the reference decode takes one token per request (T calls, state
            # chained) and an fp32 state (a bf16 state is widened)
            cur, outs = ref_state, []
            for t in range(Tdec):
                sl = slice(t, t + 1)
                o_t, cur = dec_mod.run(dec["q"][:, sl].contiguous(), dec["k"][:, sl].contiguous(),
                                       dec["v"][:, sl].contiguous(), cur, A_log,
                                       dec["a"][:, sl].contiguous(), dt_bias,
                                       dec["b"][:, sl].contiguous(), None)
                outs.append(o_t)
            keep["dec"] = (torch.cat(outs, 1), cur)
        if record:
            ev["d"].append(torch.cuda.Event(enable_timing=True))
            ev["d"][-1].record(stream)
        if pre is not None:
            keep["pre"] = pre_mod.run(pre["q"], pre["k"], pre["v"], pre["h0"], A_log, pre["a"],
                                      dt_bias, pre["b"], pre["cu"], None)
        if record:
            ev["p"].append(torch.cuda.Event(enable_timing=True))
            ev["p"][-1].record(stream)

    for _ in range(max(3, args.warmup)):
        step(False)
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(True, 0)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(args.steps):
        step(True)
    t1.record(stream)
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    ms = t0.elapsed_time(t1) / args.steps
    d_ms = float(np.mean([a.elapsed_time(b) for a, b in zip(ev["s"], ev["d"])]))
    p_ms = float(np.mean([a.elapsed_time(b) for a, b in zip(ev["d"], ev["p"])]))
    total = wl["decode_batch"] * Tdec + (pre["T"] if pre else 0)

    # our kernels on the same inputs (the reference decode left dec["state"] untouched)
    gdn = importlib.import_module("track-c-gdn_b200")

    def rel(x, y):
        x, y = x.float(), y.float()
        return float((x - y).norm() / y.norm().clamp_min(1e-30))

    parity = {}
    if dec is not None:
        if dec.get("bf16"):
            s = dec["state"].clone()
            o = gdn.decode.run_bf16_state(dec["q"], dec["k"], dec["v"], s, A_log, dec["a"],
                                          dt_bias, dec["b"], None)
        else:
            fn = gdn.decode.run if Tdec == 1 else gdn.decode.run_mtp
            o, s = fn(dec["q"], dec["k"], dec["v"], dec["state"], A_log, dec["a"], dt_bias,
                      dec["b"], None)
        parity["decode_out_rel_fro"] = rel(o, keep["dec"][0])
        parity["decode_state_rel_fro"] = rel(s, keep["dec"][1])
    if pre is not None:
        o, s = gdn.prefill.run(pre["q"], pre["k"], pre["v"], pre["h0"], A_log, pre["a"], dt_bias,
                               pre["b"], pre["cu"], None)
        parity["prefill_out_rel_fro"] = rel(o, keep["pre"][0])
        parity["prefill_state_rel_fro"] = rel(s, keep["pre"][1])
        # the reference's Triton output stage is not deterministic on B200 (whole 16-token
        # blocks of a few chunks differ between identical calls), so also give the median
        # per-token distance, which those blocks do not move
        tok = ((o.float() - keep["pre"][0].float()).flatten(1).norm(dim=1)
               / keep["pre"][0].float().flatten(1).norm(dim=1).clamp_min(1e-30))
        parity["prefill_out_token_rel_median"] = float(tok.median())
        parity["prefill_out_tokens_over_2pct"] = int((tok > 0.02).sum())
    result = {
        "impl": "triton-reference",
        "metric": "GDN serving throughput (decode + prefill tokens/s, max-over-ranks device time)",
        "value": total / (ms / 1e3), "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": ms, "higher_is_better": True,
        "dtype": "bf16", "data": "synthetic (seeded; same inputs as the b200 arm at N=1)",
        "config": {"workload": wl["desc"], "decode_batch": wl["decode_batch"],
                   "prefill_tokens": pre["T"] if pre else 0},
        "phases_ms": {"decode": d_ms, "prefill": p_ms},
        "clocks": clocks,
        "parity_b200_vs_triton": parity,
        "note": "reference Triton solutions (gdn_decode/gdn_prefill solution/triton/kernel.py, "
                "unmodified) through their run() entry points; device time with CUDA events",
    }
    if pre is not None:
        result["prefill"] = {"tokens_per_s": pre["T"] / (p_ms / 1e3),
                             "tflops": pre["T"] * PREFILL_FLOP_PER_TOKEN / (p_ms / 1e3) / 1e12}
    if dec is not None:
        result["decode"] = {"us_per_step": d_ms * 1e3,
                            "state_gbs": dec["B"] * (DECODE_STATE_BYTES + Tdec * DECODE_VEC_BYTES)
                            / (d_ms / 1e3) / 1e9}
    emit(result)


def main():
    global _JSON_FD
    sys.stdout.flush()
    _JSON_FD = os.dup(1)
    os.dup2(2, 1)
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference", "triton"], default="b200",
                    help="b200: this build; reference: CPU restatement of the reference path; "
                         "triton: the reference's Triton kernels staged under baseline/_ref (1 GPU)")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="c4")
    ap.add_argument("--e2e-steps", type=int, default=8)
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="device step only (profiling runs)")
    ap.add_argument("--no-triton", action="store_true",
                    help="N = 1: skip timing the reference's Triton kernels beside ours")
    ap.add_argument("--gather", choices=["peer", "nccl"], default="peer",
                    help="N > 1: kernels store results into rank 0's memory (peer) or an NCCL "
                         "gather runs after the compute (nccl)")
    ap.add_argument("--overlap", choices=["on", "off"], default="off",
                    help="run decode on a side stream next to the prefill (C4)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "b200":
        args.warmup = 3  # timing rule: at least three warm-up steps
    if WORKLOADS[args.workload].get("backward"):
        if args.impl != "b200":
            raise SystemExit("backward workloads: --impl b200 only (the reference has no backward)")
        bwd_arm(args)
    elif args.impl == "reference":
        reference_arm(args)
    elif args.impl == "triton":
        triton_arm(args)
    else:
        gpu_arm(args)


if __name__ == "__main__":
    main()
