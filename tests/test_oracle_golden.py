"""Pin the CPU oracle against golden vectors from the reference's own kernels.

The fixtures (tests/golden/*.npz) were produced by running the reference
Triton solutions (make_golden.py).  Three restatements are checked:
  * decode (gdn_oracle.c) must reproduce the reference decode to fp32 rounding;
  * the chunked numpy restatement must reproduce the reference prefill to
    within a bf16 rounding flip (it is bit-exact on the build machine);
  * the fp32 token recurrence (gdn_oracle.c) -- the definition's semantics --
    must agree with the reference prefill within the reference's own chunked
    error (measured 1.5-4e-3 relative on state, <=2 bf16 ulps on outputs).
"""
import numpy as np
import pytest

import cases
import golden_io
import oracle
from cases import bits_to_f32


@pytest.mark.parametrize("name", golden_io.names("decode"))
def test_decode_oracle_matches_reference(name):
    kind, inp, scale, z = golden_io.load(name)
    out, state = oracle.decode(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"],
                               inp["a"], inp["dt_bias"], inp["b"], scale)
    e_out, omax, e_proj, e_sl = golden_io.compare(z, out, state)
    # tolerance: 1 bf16 ulp at the output's magnitude; fp32 rounding on state
    assert e_out <= omax * 2.0 ** -8, (e_out, omax)
    assert e_proj < 1e-6 and e_sl < 1e-6, (e_proj, e_sl)


@pytest.mark.parametrize("name", golden_io.names("prefill"))
def test_chunked_oracle_matches_reference(name):
    kind, inp, scale, z = golden_io.load(name)
    f = bits_to_f32
    out, state = oracle.prefill_chunked(f(inp["q"]), f(inp["k"]), f(inp["v"]), inp["state"],
                                        inp["A_log"], f(inp["a"]), inp["dt_bias"], f(inp["b"]),
                                        inp["cu_seqlens"], scale)
    e_out, omax, e_proj, e_sl = golden_io.compare(z, out, state)
    # tolerance: a bf16 rounding flip of an intermediate (BLAS summation order
    # may differ between machines); an algorithmic deviation shows up as >=1e-3
    assert e_out <= max(omax, 1e-3) * 2.0 ** -7, (e_out, omax)
    assert e_proj < 2e-4 and e_sl < 2e-4, (e_proj, e_sl)


@pytest.mark.parametrize("name", golden_io.names("prefill"))
def test_recurrent_oracle_within_reference_error(name):
    kind, inp, scale, z = golden_io.load(name)
    out, state = oracle.prefill(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"],
                                inp["a"], inp["dt_bias"], inp["b"], inp["cu_seqlens"], scale)
    e_out, omax, e_proj, e_sl = golden_io.compare(z, out, state)
    # tolerance: the reference's own chunked-bf16 error vs the fp32 recurrence
    assert e_out <= 1e-3 + 1e-2 * omax, (e_out, omax)
    assert e_proj < 1e-2 and e_sl < 1e-2, (e_proj, e_sl)


def test_empty_sequence_keeps_initial_state():
    """A zero-length sequence returns its initial state unchanged (reference
    h-kernel: NT == 0 stores h0 as the final state)."""
    kind, inp, scale, z = golden_io.load("prefill_empty_seqs_h0")
    _, state = oracle.prefill(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"],
                              inp["a"], inp["dt_bias"], inp["b"], inp["cu_seqlens"], scale)
    np.testing.assert_array_equal(state[0], inp["state"][0])
    np.testing.assert_array_equal(state[2], inp["state"][2])
    np.testing.assert_array_equal(z["state_slice_first"], inp["state"][0, 0])


def test_chunked_equals_recurrence_in_exact_arithmetic():
    """Property: without bf16 rounding the chunk form is an exact
    re-association of the recurrence (checked through the recurrence vs the
    chunked oracle on a small case: their gap is the bf16 rounding only)."""
    import cases
    inp = cases.prefill_inputs(seed=99, lens=[5, 64, 70], with_state=True)
    f = bits_to_f32
    o1, s1 = oracle.prefill(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"], inp["a"],
                            inp["dt_bias"], inp["b"], inp["cu_seqlens"])
    o2, s2 = oracle.prefill_chunked(f(inp["q"]), f(inp["k"]), f(inp["v"]), inp["state"],
                                    inp["A_log"], f(inp["a"]), inp["dt_bias"], f(inp["b"]),
                                    inp["cu_seqlens"])
    assert np.abs(o1 - o2).max() < 2e-3
    assert np.linalg.norm(s1 - s2) / np.linalg.norm(s1) < 1e-2


def test_oracle_multi_token_decode_is_repeated_single_steps():
    """decode_mtp (T steps per request) equals T single decode calls fed each
    other's states, and its T = 1 case equals decode."""
    inp = cases.decode_inputs(seed=11, B=3, with_state=True)
    rng = np.random.default_rng(12)
    T = 3
    q = np.repeat(inp["q"], T, axis=1)
    k = np.repeat(inp["k"], T, axis=1)
    v = np.repeat(inp["v"], T, axis=1)
    a = rng.integers(0x3e00, 0x3f80, size=(3, T, 8)).astype(np.uint16)
    b = rng.integers(0x3e00, 0x3f80, size=(3, T, 8)).astype(np.uint16)
    out, fin, states = oracle.decode_mtp(q, k, v, inp["state"], inp["A_log"], a, inp["dt_bias"], b)
    st = inp["state"]
    for t in range(T):
        o, st = oracle.decode(q[:, t:t + 1], k[:, t:t + 1], v[:, t:t + 1], st, inp["A_log"],
                              a[:, t:t + 1], inp["dt_bias"], b[:, t:t + 1])
        np.testing.assert_array_equal(out[:, t], o[:, 0])
        np.testing.assert_array_equal(states[:, t], st)
    np.testing.assert_array_equal(fin, st)
    o1, s1, _ = oracle.decode_mtp(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"],
                                  inp["a"], inp["dt_bias"], inp["b"])
    o0, s0 = oracle.decode(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"], inp["a"],
                           inp["dt_bias"], inp["b"])
    np.testing.assert_array_equal(o1[:, 0], o0[:, 0])
    np.testing.assert_array_equal(s1, s0)
