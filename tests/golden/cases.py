"""Seeded input generators and digests shared by the golden-vector script and tests.

Inputs follow the value distributions of the benchmark configs: q/k
L2-normalised randn, v randn, state randn*0.02, A_log ~ U(0, 2.7),
a, b ~ N(0, 1), dt_bias ~ N(0, 0.1), all drawn from numpy's PCG64 so that
fixtures can be regenerated bit-for-bit.  bf16 tensors are carried as uint16
bit patterns (round-to-nearest-even from float32).
"""
from __future__ import annotations

import hashlib

import numpy as np

HQK, HV, D = 4, 8, 128


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def bits_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.asarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def _normed(rng, shape):
    x = rng.standard_normal(shape, dtype=np.float32)
    return x / np.maximum(np.linalg.norm(x, axis=-1, keepdims=True), 1e-12)


def sha(x: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(x).tobytes()).hexdigest()


def decode_inputs(seed: int, B: int, with_state: bool = True, gate_scale: float = 1.0):
    rng = np.random.default_rng(seed)
    inp = {
        "q": to_bf16_bits(_normed(rng, (B, 1, HQK, D))),
        "k": to_bf16_bits(_normed(rng, (B, 1, HQK, D))),
        "v": to_bf16_bits(rng.standard_normal((B, 1, HV, D), dtype=np.float32)),
        "A_log": (rng.random(HV, dtype=np.float32) * 2.7).astype(np.float32),
        "a": to_bf16_bits(rng.standard_normal((B, 1, HV), dtype=np.float32) * gate_scale),
        "dt_bias": (rng.standard_normal(HV, dtype=np.float32) * 0.1).astype(np.float32),
        "b": to_bf16_bits(rng.standard_normal((B, 1, HV), dtype=np.float32) * gate_scale),
    }
    st = (rng.standard_normal((B, HV, D, D), dtype=np.float32) * 0.02).astype(np.float32)
    inp["state"] = st if with_state else None
    return inp


def decode_mtp_inputs(seed: int, B: int, T: int, with_state: bool = True,
                      gate_scale: float = 1.0):
    """Multi-token decode inputs: the decode distributions with T tokens per
    request (q, k [B,T,4,128], v [B,T,8,128], a, b [B,T,8])."""
    rng = np.random.default_rng(seed)
    inp = {
        "q": to_bf16_bits(_normed(rng, (B, T, HQK, D))),
        "k": to_bf16_bits(_normed(rng, (B, T, HQK, D))),
        "v": to_bf16_bits(rng.standard_normal((B, T, HV, D), dtype=np.float32)),
        "A_log": (rng.random(HV, dtype=np.float32) * 2.7).astype(np.float32),
        "a": to_bf16_bits(rng.standard_normal((B, T, HV), dtype=np.float32) * gate_scale),
        "dt_bias": (rng.standard_normal(HV, dtype=np.float32) * 0.1).astype(np.float32),
        "b": to_bf16_bits(rng.standard_normal((B, T, HV), dtype=np.float32) * gate_scale),
    }
    st = (rng.standard_normal((B, HV, D, D), dtype=np.float32) * 0.02).astype(np.float32)
    inp["state"] = st if with_state else None
    return inp


def prefill_inputs(seed: int, lens, with_state: bool = True, gate_scale: float = 1.0):
    rng = np.random.default_rng(seed)
    T = int(sum(lens))
    N = len(lens)
    cu = np.zeros(N + 1, np.int64)
    cu[1:] = np.cumsum(np.asarray(lens, np.int64))
    inp = {
        "q": to_bf16_bits(_normed(rng, (T, HQK, D))),
        "k": to_bf16_bits(_normed(rng, (T, HQK, D))),
        "v": to_bf16_bits(rng.standard_normal((T, HV, D), dtype=np.float32)),
        "A_log": (rng.random(HV, dtype=np.float32) * 2.7).astype(np.float32),
        "a": to_bf16_bits(rng.standard_normal((T, HV), dtype=np.float32) * gate_scale),
        "dt_bias": (rng.standard_normal(HV, dtype=np.float32) * 0.1).astype(np.float32),
        "b": to_bf16_bits(rng.standard_normal((T, HV), dtype=np.float32) * gate_scale),
        "cu_seqlens": cu,
    }
    st = (rng.standard_normal((N, HV, D, D), dtype=np.float32) * 0.02).astype(np.float32)
    inp["state"] = st if with_state else None
    return inp


_PROJ = None


def state_digest(S: np.ndarray) -> dict:
    """Size-independent summary of a [..., 128, 128] state: row sums and a fixed
    4-column random projection of every row."""
    global _PROJ
    if _PROJ is None:
        _PROJ = np.random.default_rng(12345).standard_normal((D, 4)).astype(np.float64)
    S64 = np.asarray(S, np.float64)
    return {"rowsum": S64.sum(-1), "proj": S64 @ _PROJ}


# Golden cases: name -> (kind, kwargs).  Kept small: the reference runs under
# the Triton interpreter to produce them.
DECODE_CASES = {
    # benchmark config 0 shapes: batch 16, state randn*0.02
    "decode_c0_b16": dict(seed=0, B=16, with_state=True),
    "decode_b1_nostate": dict(seed=1, B=1, with_state=False),
    "decode_b3_scale05": dict(seed=2, B=3, with_state=True, scale=0.5),
    # wide gates: a*12 pushes a+dt_bias past the softplus threshold (20) and far negative
    "decode_b2_widegates": dict(seed=3, B=2, with_state=True, gate_scale=12.0),
}

PREFILL_CASES = {
    "prefill_64": dict(seed=10, lens=[64], with_state=False),
    "prefill_128_h0": dict(seed=11, lens=[128], with_state=True),
    "prefill_70": dict(seed=12, lens=[70], with_state=False),
    "prefill_70_130_h0": dict(seed=13, lens=[70, 130], with_state=True),
    "prefill_ragged_tails_h0": dict(seed=14, lens=[1, 17, 63, 65, 127], with_state=True),
    "prefill_empty_seqs_h0": dict(seed=15, lens=[0, 40, 0, 24], with_state=True),
    "prefill_widegates_h0": dict(seed=16, lens=[96], with_state=True, gate_scale=12.0),
    "prefill_scale2": dict(seed=17, lens=[33, 64], with_state=True, scale=2.0),
}
