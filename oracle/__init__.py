"""CPU oracle for the GDN decode step and prefill recurrence.

TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline leg (and its `--impl reference` arm) may import this package; the
product path (track-c-gdn_b200/) never does, and fails loudly without its own
CUDA library instead of falling back here.

Two restatements of the reference algorithm live here:
  * gdn_oracle.c  -- fp32 decode step (reference decode kernel.py:26-79) and
                     token-by-token prefill recurrence (the semantics the
                     reference's chunked prefill kernel.py:473-1542
                     re-associates), OpenMP over (sequence, v-head) pairs;
  * chunked.py    -- numpy restatement of the reference's chunk-64 WY form
                     with its bf16 rounding points, for pinning against the
                     golden vectors.
Both are pinned against tests/golden/*.npz, produced by running the
reference's own Triton kernels (tests/golden/make_golden.py).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

from .chunked import bf16_bits_to_f32, bf16_round, prefill_chunked  # noqa: F401

_HERE = Path(__file__).resolve().parent
_SRC = _HERE / "gdn_oracle.c"
_LIB_PATH = _HERE / "_build" / "libgdn_oracle.so"
_lib = None

HQK, HV, D = 4, 8, 128


def build(force: bool = False) -> Path:
    """Compile gdn_oracle.c into oracle/_build/libgdn_oracle.so (gcc, OpenMP)."""
    if _LIB_PATH.exists() and not force and _LIB_PATH.stat().st_mtime >= _SRC.stat().st_mtime:
        return _LIB_PATH
    _LIB_PATH.parent.mkdir(parents=True, exist_ok=True)
    tmp = _LIB_PATH.with_suffix(f".so.tmp{os.getpid()}")
    cmd = ["gcc", "-O3", "-march=x86-64-v3", "-fopenmp", "-shared", "-fPIC",
           "-o", str(tmp), str(_SRC), "-lm"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, _LIB_PATH)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(str(build()))
        P = ctypes.c_void_p
        lib.gdn_oracle_decode.argtypes = [ctypes.c_int, P, P, P, P, P, P, P, P,
                                          ctypes.c_float, P, P, ctypes.c_int]
        lib.gdn_oracle_decode.restype = None
        lib.gdn_oracle_prefill.argtypes = [ctypes.c_int, P, P, P, P, P, P, P, P, P,
                                           ctypes.c_float, P, P, ctypes.c_int]
        lib.gdn_oracle_prefill.restype = None
        _lib = lib
    return _lib


def _ptr(x):
    return None if x is None else x.ctypes.data_as(ctypes.c_void_p)


def _u16(x):
    x = np.ascontiguousarray(x)
    assert x.dtype == np.uint16, f"bf16 inputs are passed as uint16 bit patterns, got {x.dtype}"
    return x


def _f32(x):
    return None if x is None else np.ascontiguousarray(x, dtype=np.float32)


def default_threads() -> int:
    return len(os.sched_getaffinity(0))


def decode(q, k, v, state, A_log, a, dt_bias, b, scale=None, nthreads=None):
    """One decode step.  q,k: [B,1,4,128] u16; v: [B,1,8,128] u16;
    state: [B,8,128,128] f32 or None; a,b: [B,1,8] u16.
    Returns (out [B,1,8,128] f32, new_state [B,8,128,128] f32)."""
    lib = _load()
    q, k, v, a, b = map(_u16, (q, k, v, a, b))
    B = q.shape[0]
    if scale is None or float(scale) == 0.0:
        scale = 1.0 / np.sqrt(D)
    state = _f32(state)
    out = np.empty((B, 1, HV, D), np.float32)
    new_state = np.empty((B, HV, D, D), np.float32)
    lib.gdn_oracle_decode(B, _ptr(q), _ptr(k), _ptr(v), _ptr(state), _ptr(_f32(A_log)),
                          _ptr(a), _ptr(_f32(dt_bias)), _ptr(b), float(scale),
                          _ptr(out), _ptr(new_state), nthreads or default_threads())
    return out, new_state


def decode_mtp(q, k, v, state, A_log, a, dt_bias, b, scale=None, nthreads=None):
    """T decode steps per request, applied in order (the reference decode step,
    gdn_decode_qk4_v8_d128_k_last/solution/triton/kernel.py:26-79, once per
    token).  q,k: [B,T,4,128] u16; v: [B,T,8,128] u16; a,b: [B,T,8] u16;
    state [B,8,128,128] f32 or None.  Returns (out [B,T,8,128] f32,
    final state [B,8,128,128] f32, states after each token [B,T,8,128,128] f32)."""
    q, k, v, a, b = map(_u16, (q, k, v, a, b))
    B, T = q.shape[0], q.shape[1]
    st = None if state is None else _f32(state)
    outs, states = [], []
    for t in range(T):
        o, st = decode(q[:, t:t + 1], k[:, t:t + 1], v[:, t:t + 1], st, A_log,
                       a.reshape(B, T, HV)[:, t:t + 1], dt_bias, b.reshape(B, T, HV)[:, t:t + 1],
                       scale, nthreads)
        outs.append(o[:, 0])
        states.append(st)
    if T == 0:
        return (np.zeros((B, 0, HV, D), np.float32),
                np.zeros((B, HV, D, D), np.float32) if st is None else st,
                np.zeros((B, 0, HV, D, D), np.float32))
    return np.stack(outs, 1), st, np.stack(states, 1)


def prefill(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, scale=None, nthreads=None):
    """Prefill recurrence.  q,k: [T,4,128] u16; v: [T,8,128] u16;
    state: [N,8,128,128] f32 or None; a,b: [T,8] u16; cu_seqlens int64 [N+1].
    Returns (out [T,8,128] f32, final_state [N,8,128,128] f32)."""
    lib = _load()
    q, k, v, a, b = map(_u16, (q, k, v, a, b))
    cu = np.ascontiguousarray(cu_seqlens, dtype=np.int64)
    N = cu.shape[0] - 1
    T = q.shape[0]
    assert int(cu[-1]) == T
    if scale is None or float(scale) == 0.0:
        scale = 1.0 / np.sqrt(D)
    out = np.empty((T, HV, D), np.float32)
    final = np.empty((N, HV, D, D), np.float32)
    lib.gdn_oracle_prefill(N, _ptr(cu), _ptr(q), _ptr(k), _ptr(v), _ptr(_f32(state)),
                           _ptr(_f32(A_log)), _ptr(a), _ptr(_f32(dt_bias)), _ptr(b),
                           float(scale), _ptr(out), _ptr(final), nthreads or default_threads())
    return out, final
