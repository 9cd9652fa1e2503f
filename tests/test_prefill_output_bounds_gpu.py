"""Output bounds of the prefill scan.

A full 64-token chunk leaves the scan as one TMA store of its [64 t x 128 v]
tile per v-head; a tail chunk (fewer tokens) stores only its first L tokens
directly.  The output here is a view into a larger buffer whose guard rows
before and after hold a NaN sentinel: every output row must be written (no
sentinel left inside), nothing outside [0, T) may change, and the values must
equal those of `run` (which allocates its own output) bit for bit.  Cases:
full chunks only, tails of 1 and 63 tokens, T a multiple of 64 with a tail
in the middle, and the segmented evaluation (one long sequence; 16
sequences).
"""
import pytest
import torch

from gpu_util import device_prefill_inputs

pytestmark = pytest.mark.gpu

GUARD = 64  # rows of sentinel before and after the output
SENTINEL = 0x7FC1  # a quiet NaN in bf16


@pytest.fixture(autouse=True)
def _clean_status(gdn):
    gdn._native.read_device_status()
    yield
    assert gdn._native.read_device_status() == 0


@pytest.mark.parametrize("lens", [
    [64], [128, 64], [64, 1, 63, 65, 200], [100, 28, 64, 64], [4096],
    [300, 700, 1000, 2000, 64, 128, 65, 999, 1500, 800, 256, 512, 640, 90, 1, 3000],
])
def test_output_rows_written_exactly(gdn, lens):
    args, _ = device_prefill_inputs(lens, with_state=True, seed=sum(lens) % 1000 + 7)
    q, k, v, h0, A_log, a, dt, b, cu = args
    T, N = q.shape[0], cu.numel() - 1
    buf = torch.full((T + 2 * GUARD, 8, 128), SENTINEL, dtype=torch.int16, device="cuda")
    buf = buf.view(torch.bfloat16)
    out = buf[GUARD:GUARD + T]
    fin = torch.empty(N, 8, 128, 128, device="cuda")
    ws = gdn.prefill.alloc_workspace(T, N, q.device)
    gdn.prefill.prefill_into(q, k, v, h0, A_log, a, dt, b, cu, None, out, fin, ws)
    o_ref, s_ref = gdn.prefill.run(q, k, v, h0, A_log, a, dt, b, cu, None)
    torch.cuda.synchronize()
    raw = buf.view(torch.int16)
    assert bool((raw[:GUARD] == SENTINEL).all()), "rows before the output were written"
    assert bool((raw[GUARD + T:] == SENTINEL).all()), "rows after the output were written"
    assert not bool(torch.isnan(out.float()).any()), "an output row was not written"
    assert torch.equal(out, o_ref) and torch.equal(fin, s_ref)
