"""The prefill entry point that allocates nothing.

Some callers may not allocate device memory while they run a step -- a
plugin whose host framework owns all device memory, or a serving loop that
cannot take cudaMalloc's implicit synchronisation.  For them
gdn_prefill_qk4_v8_d128_k_last_noalloc runs the same prefill with a scratch
buffer compiled into the library instead of a caller workspace.  These tests
call it through the C ABI and check it against the regular entry point and
the fp32 recurrence oracle, on two calls in a row (the second call inherits
the first call's scratch contents); on problems whose segmented workspace
exceeds the scratch, so that the call falls back to the single-pass
evaluation; and on the size limit.  The file is named to be collected last.
"""
import ctypes

import pytest
import torch

import cases
import oracle
from gpu_util import out_err, prefill_args, rel_fro

pytestmark = pytest.mark.gpu

STATE_TOL = 5e-3  # same state tolerance as the prefill parity tests
SCRATCH = 32 << 20  # GDN_PREFILL_NOALLOC_SCRATCH_BYTES


def _noalloc(gdn, q, k, v, h0, A_log, a, dt, b, cu, out, final_state):
    return gdn._native.lib.gdn_prefill_qk4_v8_d128_k_last_noalloc(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), None if h0 is None else h0.data_ptr(),
        A_log.data_ptr(), a.data_ptr(), dt.data_ptr(), b.data_ptr(), cu.data_ptr(),
        cu.numel() - 1, q.shape[0], ctypes.c_float(0.0), out.data_ptr(),
        final_state.data_ptr(), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def _oracle(inp):
    return oracle.prefill(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"], inp["a"],
                          inp["dt_bias"], inp["b"], inp["cu_seqlens"])


def _check_case(gdn, seed, lens, with_state):
    inp = cases.prefill_inputs(seed=seed, lens=lens, with_state=with_state)
    args = prefill_args(inp)
    ref_o, ref_s = gdn.prefill.run(*args, None)
    out = torch.empty_like(ref_o)
    fs = torch.empty_like(ref_s)
    st = _noalloc(gdn, *args, out, fs)
    assert st == 0, gdn._native.lib.gdn_b200_status_string(st)
    torch.cuda.synchronize()
    assert out_err(out, ref_o.float().cpu().numpy()) <= 1.0
    assert rel_fro(fs.cpu().numpy(), ref_s.cpu().numpy()) < STATE_TOL
    ro, rs = _oracle(inp)
    assert out_err(out, ro) <= 1.0
    assert rel_fro(fs.cpu().numpy(), rs) < STATE_TOL
    return out, fs


def test_noalloc_matches_workspace_entry_point_twice(gdn):
    gdn._native.read_device_status()
    # two calls in a row with different shapes: the second runs on scratch
    # left over from the first
    for seed, lens, with_state in ((301, [17, 64, 150], True), (302, [700, 5, 129, 64], False)):
        _check_case(gdn, seed, lens, with_state)
    assert gdn._native.read_device_status() == 0


@pytest.mark.parametrize("lens", [[15_808], [7000, 7000]])
def test_noalloc_falls_back_to_single_pass_beyond_segmented_scratch(gdn, lens):
    """The segmented evaluation's workspace for these sizes exceeds the
    scratch but the single-pass one fits (T + 64 N <= 15,872; T = 15,808 for
    one sequence leaves a few tens of KB): the call must run single-pass and
    agree with the regular (segmented) entry point and the oracle."""
    T, N = sum(lens), len(lens)
    assert gdn._native.prefill_kernel_launches(T, N) == 5          # regular call: segmented
    assert gdn.prefill.workspace_bytes(T, N) > SCRATCH
    assert T + 64 * N <= 15_872
    gdn._native.read_device_status()
    _check_case(gdn, 310 + N, lens, True)
    assert gdn._native.read_device_status() == 0


def test_noalloc_rejects_problems_beyond_its_scratch(gdn):
    inp = cases.prefill_inputs(seed=303, lens=[64], with_state=False)
    q, k, v, h0, A_log, a, dt, b, cu = prefill_args(inp)
    out = torch.empty(64, 8, 128, dtype=torch.bfloat16, device="cuda")
    fs = torch.empty(1, 8, 128, 128, dtype=torch.float32, device="cuda")
    lib = gdn._native.lib
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # claim 20,000 tokens: needs more than the 32 MiB built-in scratch
    st = lib.gdn_prefill_qk4_v8_d128_k_last_noalloc(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), None, A_log.data_ptr(), a.data_ptr(),
        dt.data_ptr(), b.data_ptr(), cu.data_ptr(), 1, 20000, ctypes.c_float(0.0),
        out.data_ptr(), fs.data_ptr(), stream)
    assert st == 8  # GDN_ERR_TOO_LARGE, nothing launched
    assert b"no-allocation" in lib.gdn_b200_status_string(st)
    assert gdn.prefill.workspace_bytes(20000, 1) > SCRATCH
