"""Parity at the benchmark configurations' full sizes, token by token, against
the fp32 recurrence oracle (oracle/gdn_oracle.c, pinned to the reference's
golden vectors).

  * C3: 32 ragged sequences, lengths U{17..3000} (the benchmark's seeded
    draw), initial states randn*0.02;
  * C4 prefill: 256 sequences, lengths U{512..8192} (1,145,085 tokens), zero
    initial state -- the segmentless single-pass scan at full size;
  * decode at B = 1024 and B = 4096 (the C1 sweep's top and the C4 decode
    batch): every request.

Tolerances are the ones the other parity tests state: every output element
|d| <= 2e-3 + 1e-2 |ref| against the fp32 recurrence; final states within
5e-3 relative Frobenius (prefill, per sequence as well as overall) and 1e-5
(decode, both fp32 evaluations of the same step).  The oracle runs on all
host threads, one group of sequences at a time so host memory stays bounded.
"""
import numpy as np
import pytest
import torch

import cases
import oracle
from gpu_util import (bf16_host_bits, decode_args, device_prefill_inputs, out_err, out_err_np,
                      rel_fro)

pytestmark = pytest.mark.gpu

STATE_TOL = 5e-3


@pytest.fixture(autouse=True)
def _clean_status(gdn):
    gdn._native.read_device_status()
    yield
    assert gdn._native.read_device_status() == 0


def _lengths(config):
    # the benchmark's seeded length draws (bench.py prefill_lengths)
    if config == "c3":
        return np.random.default_rng(3).integers(17, 3001, size=32)
    return np.random.default_rng(4).integers(512, 8193, size=256)


def _check_prefill_against_oracle(out_bits, fin, host, group_tokens=160_000):
    """Every token of `out_bits` (bf16 bits [T,8,128]) and every final state
    of `fin` ([N,8,128,128] fp32) against the oracle, in sequence groups."""
    cu = host["cu_seqlens"]
    N = len(cu) - 1
    worst_out, worst_seq, num = 0.0, 0.0, 0.0
    den = 0.0
    n0 = 0
    while n0 < N:
        n1 = n0 + 1
        while n1 < N and cu[n1 + 1] - cu[n0] <= group_tokens:
            n1 += 1
        lo, hi = int(cu[n0]), int(cu[n1])
        sub_cu = cu[n0:n1 + 1] - cu[n0]
        st = None if host["state"] is None else host["state"][n0:n1]
        ro, rs = oracle.prefill(host["q"][lo:hi], host["k"][lo:hi], host["v"][lo:hi], st,
                                host["A_log"], host["a"][lo:hi], host["dt_bias"],
                                host["b"][lo:hi], sub_cu)
        o = cases.bits_to_f32(out_bits[lo:hi])
        worst_out = max(worst_out, out_err_np(o, ro))
        got = fin[n0:n1]
        for i in range(n1 - n0):
            worst_seq = max(worst_seq, rel_fro(got[i], rs[i]))
        num += float(np.sum((got.astype(np.float64) - rs) ** 2))
        den += float(np.sum(rs.astype(np.float64) ** 2))
        n0 = n1
    return worst_out, worst_seq, float(np.sqrt(num / max(den, 1e-300)))


@pytest.mark.parametrize("config", ["c3", "c4"])
def test_prefill_full_config_every_token_matches_recurrence(gdn, config):
    lengths = _lengths(config)
    args, host = device_prefill_inputs(lengths, with_state=(config == "c3"), seed=33 + len(lengths))
    launches = gdn._native.prefill_kernel_launches(int(lengths.sum()), len(lengths))
    o, s = gdn.prefill.run(*args, None)
    torch.cuda.synchronize()
    out_bits = bf16_host_bits(o)
    fin = s.cpu().numpy()
    del o, s
    worst_out, worst_seq, overall = _check_prefill_against_oracle(out_bits, fin, host)
    print(f"{config}: T={int(lengths.sum())} N={len(lengths)} launches={launches} "
          f"out ratio max {worst_out:.3f}, state rel fro worst sequence {worst_seq:.2e}, "
          f"overall {overall:.2e}")
    assert worst_out <= 1.0, worst_out
    assert worst_seq < STATE_TOL, worst_seq
    assert overall < STATE_TOL, overall


@pytest.mark.parametrize("B", [1024, 4096])
def test_decode_full_batch_every_request_matches_oracle(gdn, B):
    inp = cases.decode_inputs(seed=900 + B, B=B)
    args = decode_args(inp)
    o, s = gdn.decode.run(*args, None)
    torch.cuda.synchronize()
    ro, rs = oracle.decode(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"], inp["a"],
                           inp["dt_bias"], inp["b"])
    assert out_err(o, ro) <= 1.0
    got = s.cpu().numpy()
    per_req = [rel_fro(got[i], rs[i]) for i in range(B)]
    print(f"decode B={B}: out ratio {out_err(o, ro):.3f}, state worst request {max(per_req):.2e}")
    assert max(per_req) < 1e-5
    # the in-place serving form on the same inputs: identical results
    st = args[3].clone()
    o2 = gdn.decode.run_inplace(args[0], args[1], args[2], st, *args[4:], None)
    assert torch.equal(o2, o) and torch.equal(st, s)
