"""Multi-token decode (speculative verify / MTP) on the GPU, through the C ABI.

T tokens per request must equal T single-token decode steps:
  * bit for bit against this library's single-token kernel applied T times
    (same fp32 arithmetic in the same order), outputs, the state after every
    token and the final state;
  * within the decode tolerances against the fp32 oracle applied T times:
    outputs |d| <= 2e-3 + 1e-2 |ref|, final state relative Frobenius <= 1e-5.
"""
import ctypes

import numpy as np
import pytest
import torch

import cases
import oracle
from gpu_util import bf16_dev, f32_dev, out_err, rel_fro

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _clean_status(gdn):
    gdn._native.read_device_status()
    yield
    assert gdn._native.read_device_status() == 0


def _dev(inp):
    return (bf16_dev(inp["q"]), bf16_dev(inp["k"]), bf16_dev(inp["v"]), f32_dev(inp["state"]),
            f32_dev(inp["A_log"]), bf16_dev(inp["a"]), f32_dev(inp["dt_bias"]), bf16_dev(inp["b"]))


@pytest.mark.parametrize("B,T,with_state", [
    (1, 1, True), (3, 2, True), (16, 4, False), (300, 7, True), (64, 16, True), (2, 64, True),
])
def test_mtp_equals_sequential_single_steps(gdn, B, T, with_state):
    inp = cases.decode_mtp_inputs(seed=100 * B + T, B=B, T=T, with_state=with_state)
    q, k, v, st, A_log, a, dt, b = _dev(inp)
    o, s, inter = gdn.decode.run_mtp(q, k, v, st, A_log, a, dt, b, None, return_intermediate=True)
    cur = st
    for t in range(T):
        sl = slice(t, t + 1)
        ot, cur = gdn.decode.run(q[:, sl].contiguous(), k[:, sl].contiguous(),
                                 v[:, sl].contiguous(), cur, A_log, a[:, sl].contiguous(), dt,
                                 b[:, sl].contiguous(), None)
        assert torch.equal(o[:, t], ot[:, 0]), t
        assert torch.equal(inter[:, t], cur), t
    assert torch.equal(s, cur)


@pytest.mark.parametrize("B,T", [(4, 3), (33, 5)])
def test_mtp_matches_oracle(gdn, B, T):
    inp = cases.decode_mtp_inputs(seed=7 * B + T, B=B, T=T, with_state=True)
    o, s = gdn.decode.run_mtp(*_dev(inp), None)
    torch.cuda.synchronize()
    ro, rs, _ = oracle.decode_mtp(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"],
                                  inp["a"], inp["dt_bias"], inp["b"])
    assert out_err(o, ro) <= 1.0
    assert rel_fro(s.cpu().numpy(), rs) < 1e-5


def test_mtp_in_place_equals_out_of_place(gdn):
    inp = cases.decode_mtp_inputs(seed=5, B=24, T=4, with_state=True)
    q, k, v, st, A_log, a, dt, b = _dev(inp)
    o_ref, s_ref = gdn.decode.run_mtp(q, k, v, st, A_log, a, dt, b, 0.1)
    out = torch.empty_like(o_ref)
    gdn.decode.decode_mtp_into(q, k, v, st, A_log, a, dt, b, 0.1, out, st)  # new_state = state
    torch.cuda.synchronize()
    assert torch.equal(out, o_ref) and torch.equal(st, s_ref)


def test_mtp_rejects_bad_token_counts(gdn):
    inp = cases.decode_mtp_inputs(seed=6, B=2, T=2, with_state=True)
    q, k, v, st, A_log, a, dt, b = _dev(inp)
    lib = gdn._native.lib
    out = torch.empty(2, 2, 8, 128, dtype=torch.bfloat16, device="cuda")
    ns = torch.empty_like(st)
    args = (q.data_ptr(), k.data_ptr(), v.data_ptr(), st.data_ptr(), A_log.data_ptr(),
            a.data_ptr(), dt.data_ptr(), b.data_ptr(), ctypes.c_float(0.0), 2)
    for T in (0, 65):
        assert lib.gdn_decode_mtp_qk4_v8_d128_k_last(*args, T, out.data_ptr(), ns.data_ptr(),
                                                     None, None) == 2
