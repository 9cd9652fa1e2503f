"""Prefill parity on the GPU: the sm_100a chunk kernels (through the C ABI)
against the fp32 recurrence oracle, the reference's golden vectors, and
size-independent properties at full sizes.

Tolerances (stated per the benchmark definition):
  * outputs (bf16): |d| <= 2e-3 + 1e-2 |ref| against the fp32 recurrence;
  * final state (fp32): relative Frobenius error <= 5e-3 against the fp32
    recurrence.  The reference's own chunked kernel (bf16 w/u/h/v_new
    operands) sits at 1.5-4e-3 on these inputs (the chunked oracle, which is
    bit-exact with it, measures that gap in test_state_error_not_worse_than_reference);
    this kernel must stay within 1.5x of it.
"""
import numpy as np
import pytest
import torch

import cases
import golden_io
import oracle
from cases import bits_to_f32
from gpu_util import out_err, prefill_args, rel_fro

pytestmark = pytest.mark.gpu

STATE_TOL = 5e-3


@pytest.fixture(autouse=True)
def _clean_status(gdn):
    gdn._native.read_device_status()
    yield
    assert gdn._native.read_device_status() == 0


def _run(gdn, inp, scale=None):
    o, s = gdn.prefill.run(*prefill_args(inp), scale)
    torch.cuda.synchronize()
    return o, s


def _oracle(inp, scale=None):
    return oracle.prefill(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"], inp["a"],
                          inp["dt_bias"], inp["b"], inp["cu_seqlens"], scale)


@pytest.mark.parametrize("name", golden_io.names("prefill"))
def test_prefill_golden_cases_match_recurrence(gdn, name):
    kind, inp, scale, z = golden_io.load(name)
    o, s = _run(gdn, inp, scale)
    ro, rs = _oracle(inp, scale)
    assert out_err(o, ro) <= 1.0
    assert rel_fro(s.cpu().numpy(), rs) < STATE_TOL
    # and against the reference's own outputs (two chunked bf16 evaluations)
    e_out, omax, e_proj, e_sl = golden_io.compare(z, o.float().cpu().numpy(), s.cpu().numpy())
    assert e_out <= 4e-3 + 2e-2 * omax, (e_out, omax)
    assert e_proj < 2 * STATE_TOL and e_sl < 2 * STATE_TOL, (e_proj, e_sl)


@pytest.mark.parametrize("lens,with_state", [
    ([1], True), ([17], False), ([63], True), ([64], True), ([65], True), ([127], False),
    ([128], True), ([300], True), ([5, 64, 200, 1], True), ([1000], False),
])
def test_prefill_ragged_matches_recurrence(gdn, lens, with_state):
    inp = cases.prefill_inputs(seed=sum(lens) + len(lens), lens=lens, with_state=with_state)
    o, s = _run(gdn, inp)
    ro, rs = _oracle(inp)
    assert out_err(o, ro) <= 1.0
    assert rel_fro(s.cpu().numpy(), rs) < STATE_TOL


def test_prefill_many_sequences_wide_path(gdn):
    """N=24 sequences: one CTA per (sequence, v-head) (128-wide v-slices)."""
    rng = np.random.default_rng(3)
    lens = list(rng.integers(1, 400, size=24))
    inp = cases.prefill_inputs(seed=31, lens=lens, with_state=True)
    o, s = _run(gdn, inp)
    ro, rs = _oracle(inp)
    assert out_err(o, ro) <= 1.0
    assert rel_fro(s.cpu().numpy(), rs) < STATE_TOL


def test_prefill_config_c2_t4096(gdn):
    """Benchmark config 2: one packed sequence T=4096, zero initial state."""
    inp = cases.prefill_inputs(seed=0, lens=[4096], with_state=False)
    o, s = _run(gdn, inp)
    ro, rs = _oracle(inp)
    assert out_err(o, ro) <= 1.0
    assert rel_fro(s.cpu().numpy(), rs) < STATE_TOL


@pytest.mark.parametrize("lens,with_state", [
    ([4096], True), ([769], True), ([3000, 1500], True), ([0, 2000, 900], True),
    ([1024, 1024, 1024], False),
])
def test_segmented_evaluation_matches_recurrence(gdn, lens, with_state):
    """Few long sequences take the segmented path (segments in parallel,
    joined through their affine state maps): same tolerances as one pass.
    [769] ends in a ragged chunk inside its last segment; [0, ...] mixes in
    an empty sequence."""
    assert gdn._native.prefill_kernel_launches(sum(lens), len(lens)) == 5
    inp = cases.prefill_inputs(seed=sum(lens) + 7, lens=lens, with_state=with_state)
    o, s = _run(gdn, inp)
    ro, rs = _oracle(inp)
    assert out_err(o, ro) <= 1.0
    assert rel_fro(s.cpu().numpy(), rs) < STATE_TOL
    if lens[0] == 0 and with_state:
        np.testing.assert_array_equal(s[0].cpu().numpy(), inp["state"][0])


@pytest.mark.parametrize("lens", [[4096], [3000, 1500]])
def test_segmented_composition_with_slow_decay(gdn, lens):
    """With the benchmark gates a 256-token segment decays its state map Phi
    to zero in fp32, so the composition S(p+1) = S(p) Phi(p) + B(p) reduces
    to B(p).  Here A_log in [-5, -2] keeps the segment decay between e^-1.5
    and e^-17, so the S(p) Phi(p) products carry the state across segments
    and are checked against the recurrence."""
    assert gdn._native.prefill_kernel_launches(sum(lens), len(lens)) == 5
    inp = cases.prefill_inputs(seed=sum(lens) + 11, lens=lens, with_state=True)
    inp["A_log"] = (np.random.default_rng(5).random(8, dtype=np.float32) * 3.0 - 5.0).astype(
        np.float32)
    o, s = _run(gdn, inp)
    ro, rs = _oracle(inp)
    f = bits_to_f32
    _, cs = oracle.prefill_chunked(f(inp["q"]), f(inp["k"]), f(inp["v"]), inp["state"],
                                   inp["A_log"], f(inp["a"]), inp["dt_bias"], f(inp["b"]),
                                   inp["cu_seqlens"])
    assert out_err(o, ro) <= 1.0
    assert rel_fro(s.cpu().numpy(), rs) < STATE_TOL
    assert rel_fro(s.cpu().numpy(), rs) <= 1.5 * rel_fro(cs, rs) + 1e-4


def test_single_pass_with_slow_decay(gdn):
    """Ragged sequences on the single-pass scan with A_log in [-5, -2]: the
    state carried from chunk to chunk (and h0) stays large, so the inter-chunk
    update of the scan is exercised, not only the intra-chunk terms."""
    lens = [700, 5, 129, 64, 1000]
    assert gdn._native.prefill_kernel_launches(sum(lens), len(lens)) == 3
    inp = cases.prefill_inputs(seed=sum(lens) + 13, lens=lens, with_state=True)
    inp["A_log"] = (np.random.default_rng(6).random(8, dtype=np.float32) * 3.0 - 5.0).astype(
        np.float32)
    o, s = _run(gdn, inp)
    ro, rs = _oracle(inp)
    f = bits_to_f32
    _, cs = oracle.prefill_chunked(f(inp["q"]), f(inp["k"]), f(inp["v"]), inp["state"],
                                   inp["A_log"], f(inp["a"]), inp["dt_bias"], f(inp["b"]),
                                   inp["cu_seqlens"])
    assert out_err(o, ro) <= 1.0
    assert rel_fro(s.cpu().numpy(), rs) <= 1.5 * rel_fro(cs, rs) + 1e-4


def test_segmented_state_error_not_worse_than_reference(gdn):
    inp = cases.prefill_inputs(seed=42, lens=[1500], with_state=True)
    assert gdn._native.prefill_kernel_launches(1500, 1) == 5
    o, s = _run(gdn, inp)
    ro, rs = _oracle(inp)
    f = bits_to_f32
    _, cs = oracle.prefill_chunked(f(inp["q"]), f(inp["k"]), f(inp["v"]), inp["state"],
                                   inp["A_log"], f(inp["a"]), inp["dt_bias"], f(inp["b"]),
                                   inp["cu_seqlens"])
    assert rel_fro(s.cpu().numpy(), rs) <= 1.5 * rel_fro(cs, rs) + 1e-4


def test_state_error_not_worse_than_reference(gdn):
    """The kernel's state error vs the exact recurrence stays within 1.5x of
    the reference algorithm's own (chunked oracle == reference kernel)."""
    inp = cases.prefill_inputs(seed=41, lens=[70, 130, 257], with_state=True)
    o, s = _run(gdn, inp)
    ro, rs = _oracle(inp)
    f = bits_to_f32
    _, cs = oracle.prefill_chunked(f(inp["q"]), f(inp["k"]), f(inp["v"]), inp["state"],
                                   inp["A_log"], f(inp["a"]), inp["dt_bias"], f(inp["b"]),
                                   inp["cu_seqlens"])
    assert rel_fro(s.cpu().numpy(), rs) <= 1.5 * rel_fro(cs, rs) + 1e-4


def test_resume_is_bit_exact_on_chunk_boundary(gdn):
    """prefill(a + b) == prefill(a) then prefill(b) from its final state, bit
    for bit, when a is a multiple of 64 (same chunking)."""
    inp = cases.prefill_inputs(seed=51, lens=[192 + 77], with_state=True)
    q, k, v, h0, A_log, a, dt, b, cu = prefill_args(inp)
    o_full, s_full = gdn.prefill.run(q, k, v, h0, A_log, a, dt, b, cu, None)
    cut = 192
    cu1 = torch.tensor([0, cut], dtype=torch.int64, device="cuda")
    cu2 = torch.tensor([0, 269 - cut], dtype=torch.int64, device="cuda")
    o1, s1 = gdn.prefill.run(q[:cut], k[:cut], v[:cut], h0, A_log, a[:cut], dt, b[:cut], cu1, None)
    o2, s2 = gdn.prefill.run(q[cut:].contiguous(), k[cut:].contiguous(), v[cut:].contiguous(), s1,
                             A_log, a[cut:].contiguous(), dt, b[cut:].contiguous(), cu2, None)
    assert torch.equal(torch.cat([o1, o2]), o_full)
    assert torch.equal(s2, s_full)


def test_resume_off_boundary_within_tolerance(gdn):
    inp = cases.prefill_inputs(seed=52, lens=[300], with_state=True)
    q, k, v, h0, A_log, a, dt, b, cu = prefill_args(inp)
    o_full, s_full = gdn.prefill.run(q, k, v, h0, A_log, a, dt, b, cu, None)
    cut = 100
    cu1 = torch.tensor([0, cut], dtype=torch.int64, device="cuda")
    cu2 = torch.tensor([0, 300 - cut], dtype=torch.int64, device="cuda")
    o1, s1 = gdn.prefill.run(q[:cut], k[:cut], v[:cut], h0, A_log, a[:cut], dt, b[:cut], cu1, None)
    o2, s2 = gdn.prefill.run(q[cut:].contiguous(), k[cut:].contiguous(), v[cut:].contiguous(), s1,
                             A_log, a[cut:].contiguous(), dt, b[cut:].contiguous(), cu2, None)
    ro, rs = _oracle(inp)
    assert out_err(torch.cat([o1, o2]), ro) <= 1.0
    assert rel_fro(s2.cpu().numpy(), rs) < STATE_TOL


def test_sequence_independence(gdn):
    """A sequence's outputs do not depend on its neighbours in the batch."""
    inp = cases.prefill_inputs(seed=61, lens=[50, 130, 64], with_state=True)
    q, k, v, h0, A_log, a, dt, b, cu = prefill_args(inp)
    o, s = gdn.prefill.run(q, k, v, h0, A_log, a, dt, b, cu, None)
    lo, hi = 50, 180
    cu1 = torch.tensor([0, hi - lo], dtype=torch.int64, device="cuda")
    o1, s1 = gdn.prefill.run(q[lo:hi].contiguous(), k[lo:hi].contiguous(), v[lo:hi].contiguous(),
                             h0[1:2].contiguous(), A_log, a[lo:hi].contiguous(), dt,
                             b[lo:hi].contiguous(), cu1, None)
    assert torch.equal(o[lo:hi], o1)
    assert torch.equal(s[1:2], s1)


def test_empty_sequences_return_initial_state(gdn):
    inp = cases.prefill_inputs(seed=71, lens=[0, 40, 0, 24, 0], with_state=True)
    o, s = _run(gdn, inp)
    st = s.cpu().numpy()
    for n in (0, 2, 4):
        np.testing.assert_array_equal(st[n], inp["state"][n])
    ro, rs = _oracle(inp)
    assert out_err(o, ro) <= 1.0
    assert rel_fro(st, rs) < STATE_TOL


def test_all_empty(gdn):
    inp = cases.prefill_inputs(seed=72, lens=[0, 0], with_state=True)
    o, s = _run(gdn, inp)
    assert o.shape == (0, 8, 128)
    np.testing.assert_array_equal(s.cpu().numpy(), inp["state"])


def test_inplace_state(gdn):
    inp = cases.prefill_inputs(seed=73, lens=[90, 10], with_state=True)
    q, k, v, h0, A_log, a, dt, b, cu = prefill_args(inp)
    o_ref, s_ref = gdn.prefill.run(q, k, v, h0, A_log, a, dt, b, cu, None)
    out = torch.empty_like(o_ref)
    ws = gdn.prefill.alloc_workspace(q.shape[0], 2, "cuda")
    gdn.prefill.prefill_into(q, k, v, h0, A_log, a, dt, b, cu, None, out, h0, ws)
    assert torch.equal(out, o_ref) and torch.equal(h0, s_ref)


def test_bad_cu_seqlens_sets_device_status(gdn):
    """cu_seqlens[-1] != T is caught on the device (no fault, no output)."""
    inp = cases.prefill_inputs(seed=74, lens=[64, 64], with_state=True)
    q, k, v, h0, A_log, a, dt, b, cu = prefill_args(inp)
    bad = torch.tensor([0, 64, 100], dtype=torch.int64, device="cuda")
    out = torch.empty(128, 8, 128, dtype=torch.bfloat16, device="cuda")
    fs = torch.empty_like(h0)
    ws = gdn.prefill.alloc_workspace(128, 2, "cuda")
    gdn.prefill.prefill_into(q, k, v, h0, A_log, a, dt, b, bad, None, out, fs, ws)
    assert gdn._native.read_device_status() == 1
    # the reference-compatible entry point asserts on the host, like the reference
    with pytest.raises(AssertionError):
        gdn.prefill.run(q, k, v, h0, A_log, a, dt, b, bad, None)


def test_decode_continues_prefill(gdn):
    """prefill(T) followed by one decode step == prefill(T + 1) (two kernels,
    one recurrence; decode uses the thresholded softplus, equal here)."""
    inp = cases.prefill_inputs(seed=81, lens=[129], with_state=True)
    q, k, v, h0, A_log, a, dt, b, cu = prefill_args(inp)
    o_full, s_full = gdn.prefill.run(q, k, v, h0, A_log, a, dt, b, cu, None)
    cu1 = torch.tensor([0, 128], dtype=torch.int64, device="cuda")
    _, s1 = gdn.prefill.run(q[:128], k[:128], v[:128], h0, A_log, a[:128], dt, b[:128], cu1, None)
    t = 128
    od, sd = gdn.decode.run(q[t:t + 1].view(1, 1, 4, 128), k[t:t + 1].view(1, 1, 4, 128),
                            v[t:t + 1].view(1, 1, 8, 128), s1, A_log, a[t:t + 1].view(1, 1, 8), dt,
                            b[t:t + 1].view(1, 1, 8), None)
    assert out_err(od.view(1, 8, 128), o_full[t:t + 1].float().cpu().numpy()) <= 1.0
    assert rel_fro(sd.cpu().numpy(), s_full.cpu().numpy()) < STATE_TOL


def test_repeated_back_to_back_runs_are_deterministic(gdn):
    """Eight back-to-back prefills of 48 long ragged sequences (no host sync in
    between) give bit-identical results and leave the device status clean:
    catches barrier-phase races in the pipelined scan."""
    rng = np.random.default_rng(91)
    lens = list(rng.integers(300, 3000, size=48))
    inp = cases.prefill_inputs(seed=92, lens=lens, with_state=False)
    q, k, v, h0, A_log, a, dt, b, cu = prefill_args(inp)
    T, N = q.shape[0], len(lens)
    ws = gdn.prefill.alloc_workspace(T, N, "cuda")
    outs = []
    for _ in range(8):
        o = torch.empty(T, 8, 128, dtype=torch.bfloat16, device="cuda")
        s = torch.empty(N, 8, 128, 128, dtype=torch.float32, device="cuda")
        gdn.prefill.prefill_into(q, k, v, None, A_log, a, dt, b, cu, None, o, s, ws)
        outs.append((o, s))
    torch.cuda.synchronize()
    assert gdn._native.read_device_status() == 0
    for o, s in outs[1:]:
        assert torch.equal(o, outs[0][0]) and torch.equal(s, outs[0][1])


@pytest.mark.parametrize("lens", [[300, 64, 17], [4096]])  # single-pass, segmented
def test_prefill_events_variant_times_each_kernel(gdn, lens):
    """prefill_into(..., events=...) records one event after each kernel the
    call launches (gdn_prefill_qk4_v8_d128_k_last_events) and gives the same
    results bit for bit."""
    inp = cases.prefill_inputs(seed=sum(lens) + 3, lens=lens, with_state=True)
    q, k, v, h0, A_log, a, dt, b, cu = prefill_args(inp)
    T, N = q.shape[0], len(lens)
    n = gdn._native.prefill_kernel_launches(T, N)
    ws = gdn.prefill.alloc_workspace(T, N, "cuda")
    o1 = torch.empty(T, 8, 128, dtype=torch.bfloat16, device="cuda")
    s1 = torch.empty_like(h0)
    gdn.prefill.prefill_into(q, k, v, h0, A_log, a, dt, b, cu, None, o1, s1, ws)
    start = torch.cuda.Event(enable_timing=True)
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(n)]
    o2, s2 = torch.empty_like(o1), torch.empty_like(s1)
    start.record()
    gdn.prefill.prefill_into(q, k, v, h0, A_log, a, dt, b, cu, None, o2, s2, ws, events=evs)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2) and torch.equal(s1, s2)
    times = [(start if i == 0 else evs[i - 1]).elapsed_time(evs[i]) for i in range(n)]
    assert all(t >= 0 for t in times) and sum(times) > 0, times


MANY_LENS = [3000, 1000, 700, 5000, 513, 1025, 2049, 100, 64, 65, 900, 1500, 777, 1200, 333,
             2500]


@pytest.mark.parametrize("slow_decay", [False, True])
def test_segmented_evaluation_with_many_sequences(gdn, slow_decay):
    """16 sequences, the most the segmented evaluation takes, with lengths
    from 64 to 5,000 tokens: in one call the shortest ones (at most one
    segment) run whole in pass 1 while the others are cut into two or more
    segments.  Against the fp32 recurrence, with the benchmark gates and with
    slow decay (A_log in [-5, -2]) so that the joined state maps matter."""
    lens = MANY_LENS
    assert gdn._native.prefill_kernel_launches(sum(lens), len(lens)) == 5
    inp = cases.prefill_inputs(seed=sum(lens) + 21, lens=lens, with_state=True)
    if slow_decay:
        inp["A_log"] = (np.random.default_rng(8).random(8, dtype=np.float32) * 3.0 - 5.0).astype(
            np.float32)
    o, s = _run(gdn, inp)
    ro, rs = _oracle(inp)
    assert out_err(o, ro) <= 1.0
    st = s.cpu().numpy()
    assert rel_fro(st, rs) < STATE_TOL
    assert max(rel_fro(st[i], rs[i]) for i in range(len(lens))) < STATE_TOL
